// rkv_mla_decode.cu -- MLA decode attention that reads the FP8 pages directly.
//
// The consumer of the paged rows: rsLLM's mixed attention sweep
// (crates/rsllm-models/src/dsv4/attention.rs:493-663) for one query position
// per CTA, 64 heads sharing one latent KV row per token (MQA form of MLA):
//   S = Q K^T * scale over the 576 stored lanes, softmax with the per-head sink
//   as a value-less virtual key, O = P V over the 512 latent lanes; the keys
//   are every row of the query's sequence (dense) or only the rows an index
//   list selects (the sparse mask of attention.rs:548-556).
//
// The FP8 rows are never written back as bf16: loader warps read a page's
// codes, scales and RoPE lanes with 256-bit loads, dequantise them (exactly,
// see BitScale below) straight into a 128-byte-swizzled shared-memory tile,
// and the 5th-generation tensor cores consume that tile twice -- as K
// (K-major) for S and as V (MN-major) for O:
//
//   warps 0-3  softmax: Q into TMEM once; S from TMEM, online max / exp2 /
//              row sums per head, P (bf16) into shared memory, the rare lazy
//              rescale of O, epilogue
//   warps 4-11 loaders, software-pipelined over two register buffers: the
//              loads of tile j + 1 are in flight while tile j is
//              dequantised into its stage
//   warp 12    TMEM allocation and S = Q K^T of every loaded tile
//   warp 13    O += P V of every softmaxed tile
//   warp 14    resolver: key rows to pool slots and key masks up to four
//              tiles ahead; in dense mode an L2 prefetch of each tile's page
//
// Shapes per tile (64 key rows, one page in dense mode), M = 64 heads:
//   S[64 x 64]   = Q[64 x 576] . K^T    36 MMAs of K = 16, N = 64; Q from
//                                       TMEM, K from shared memory
//   O[64 x 512] += P[64 x 64]  . V      2 x 4 MMAs of N = 256, both operands
//                                       from shared memory
// An M = 64 operand occupies 16 lanes of each 32-lane TMEM sub-partition
// (head h in lane (h % 16) + 32 (h / 16) + base).  Lanes 0-15: Q at columns
// 0-287 (bf16 pairs) and S double-buffered at 288 and 352 -- an MMA with A in
// TMEM keeps its accumulator in those same lanes.  Lanes 16-31: O, latent
// 0-255 at columns 0-255 and 256-511 at 256-511.  Keeping Q out of shared
// memory leaves room for three K/V stages (72 KB each) and P (8 KB); Q passes
// through stage 2 and P on its way into TMEM, before either is needed.
//
// Three stages keep the loads and the dequantisation ahead of the tensor
// cores.  The online softmax keeps a per-head reference maximum m and
// rescales O only when a tile's maximum exceeds it by more than 2^8 (P values
// stay <= 256 in bf16).  The final normalisation uses the same m, so the
// result is the same softmax; the denominator is the sum of the bf16-rounded
// P the tensor core multiplies, plus the sink's exp.
//
// Every wait on a barrier is bounded (1 s of %globaltimer); on a timeout the
// CTA records RKV_ERR_CUDA in the status word, drains its own MMAs, frees its
// tensor memory and returns.
#include <cmath>

#include <atomic>

#include "rkv_common.cuh"
#include "rkv_host.h"

namespace rkv {
namespace mla {

constexpr int kHeads = 64;
constexpr int kQk = 576;                      // key lanes: 512 latent + 64 RoPE
constexpr int kV = 512;                       // value lanes: the latent
constexpr int kTile = 64;                     // key rows per tile
constexpr int kAtom = 1024;                   // 8 rows x 128 B swizzle atom
constexpr int kColBytes = 8 * kAtom;          // one 64-lane column of a 64-row operand
constexpr int kOperandBytes = (kQk / 64) * kColBytes;  // 73728: 64 rows x 576 bf16
constexpr int kStages = 3;
constexpr int kSmemK0 = 0;                    // three K/V stages of 64 rows x 576 bf16
constexpr int kSmemP = kSmemK0 + kStages * kOperandBytes;  // P: 64 heads x 64 keys bf16
constexpr int kSmemBar = kSmemP + kColBytes;
constexpr int kSmemRows = kSmemBar + 336;     // slot tables: 4 x 64 x int32 (page * 64 + row, -1 = none)
constexpr int kSmemTotal = kSmemRows + 4 * 64 * 4;
constexpr int kSmemAlloc = kSmemTotal + 1024; // slack for the 1024-byte alignment
// Q arrives by bulk copies into stage 2 and P, which nothing else uses before
// tile 2 is stored: row h at q_row_off(h), 16 B further round the banks per
// row so that 16 rows read together take the minimum two wavefronts.
constexpr int kSmemQ = kSmemK0 + (kStages - 1) * kOperandBytes;
constexpr int kQRowBytes = kQk * 2;
__host__ __device__ constexpr int q_row_off(int h) {
  return (h >> 3) * (8 * kQRowBytes + 128) + (h & 7) * (kQRowBytes + 16);
}
static_assert(kSmemQ + q_row_off(kHeads - 1) + kQRowBytes <= kSmemP + kColBytes, "Q staging overruns P");
constexpr int kThreads = 480;  // warps 0-3 softmax, 4-11 loaders, 12 S issuer, 13 O issuer, 14 resolver
constexpr int kLoaders = 256;
constexpr int kQkWarp = 12, kResolverWarp = 14;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 288;               // S buffers at 288 and 352 (lanes 0-15); Q at 0-287
constexpr uint32_t kLaneO = 16u << 16;        // O in lanes 16-31 of every sub-partition, columns 0-511
constexpr float kRescaleLog2 = 8.0f;
constexpr uint64_t kTimeoutNs = 1000000000ull;

// Barrier / state offsets inside the kSmemBar block: stage barriers indexed
// by j % 3, S barriers (full, free) by j & 1, slot tables by j & 3, key
// masks by j & 15.
constexpr int kBarKFull = 0, kBarKEmpty = 24, kBarSFull = 48, kBarSFree = 64, kBarPFull = 80, kBarPvDone = 88,
              kBarDrain = 96, kBarQReady = 112, kBarTabFull = 120, kBarTabFree = 152;  // drain: S and O issuers
constexpr int kTmemSlot = 184, kAbort = 188, kBarQLoad = 192, kMask = 200;

constexpr uint32_t kIdescQK = (1u << 4) | (1u << 7) | (1u << 10) | ((64u >> 3) << 17) | ((64u >> 4) << 24);
constexpr uint32_t kIdescPV = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 16) | ((256u >> 3) << 17) | ((64u >> 4) << 24);

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for a bulk copy's barrier; it ignores the abort flag, so that a
// CTA never leaves with a copy into its shared memory still in flight.
__device__ bool mbar_wait_copy(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = now_ns();
  while (!mbar_test(bar, parity))
    if (now_ns() - t0 > kTimeoutNs) return false;
  return true;
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
// Global -> shared bulk copy (no multicast), completing on an mbarrier.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
// Bounded wait for the phase of the given parity; false on timeout or abort.
__device__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_test(bar, parity)) return true;
  const uint64_t t0 = now_ns();
  while (!mbar_test(bar, parity)) {
    if (*abort_flag) return false;
    if (now_ns() - t0 > kTimeoutNs) return false;
  }
  return true;
}

__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 128-byte-swizzle shared-memory matrix descriptor (sm_100 version field).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3fffu) | ((uint64_t)((lbo >> 4) & 0x3fffu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// Same with the A operand in tensor memory (K-major bf16 pairs per column).
__device__ __forceinline__ void mma_bf16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// One lane of a converged warp (the same lane on every call).
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile("{\n\t.reg .pred P;\n\telect.sync _|P, 0xffffffff;\n\tselp.u32 %0, 1, 0, P;\n\t}" : "=r"(pred));
  return pred != 0;
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
      "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// 16 lanes x 256 bits, 4 repetitions (32 columns): thread t holds lanes
// t / 4 (registers 4r, 4r + 1) and t / 4 + 8 (4r + 2, 4r + 3) at columns
// 8r + 2 (t % 4) and 8r + 2 (t % 4) + 1.
__device__ __forceinline__ void tmem_ld16x256(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16x256x8(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16x256(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x256b.x4.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ unsigned long long pk2(uint32_t lo, uint32_t hi) {
  return ((unsigned long long)hi << 32) | lo;
}
__device__ __forceinline__ unsigned long long mul_f32x2(unsigned long long a, unsigned long long b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// max(a, b, c) in one instruction (sm_100); NaN handling as fmaxf.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// Byte offset of 16-byte chunk `c` (8 bf16 lanes) of row `r` in a 64-row
// operand stored as 64-lane columns of 8-row swizzle atoms.
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
  return (uint32_t)((c >> 3) * kColBytes + (r >> 3) * kAtom + (r & 7) * 128 + (((c & 7) ^ (r & 7)) << 4));
}

struct Params {
  rkv_pool_view pool;
  int layer;
  const int32_t* page_table;
  int64_t pt_stride;
  const int32_t* seq_lens;
  const int32_t* seq_of_query;
  const uint16_t* q;   // bf16 [n_q][64][576]
  const int32_t* idx;  // [n_q][k] or null (dense)
  int k;
  const float* sinks;  // [64] or null
  float scale_log2;    // softmax scale * log2(e)
  int n_splits;
  float* ws_o;         // [n_q][n_splits][64][512] when n_splits > 1
  float* ws_ml;        // [n_q][n_splits][64][2]
  float* out;          // [n_q][64][512]
  uint32_t* status;
};

// Latent lane order in shared memory and in Q's TMEM copy: within every group
// of four lanes, stored order (0, 2, 1, 3).  The loaders then build each bf16
// pair straight from two code bytes: an E4M3 byte's sign and 7 magnitude
// bits placed as a bf16's sign, exponent and top mantissa bits read as
// value * 2^-120 (normal or subnormal alike), so one bf16 multiply by
// 2^(120+e) gives value * 2^e -- exact, or +-inf on overflow, the same bits
// as the f32 product rounded to bf16.  S sums over lanes in any order the MMA
// likes, so Q in the same lane order leaves it unchanged; O comes out with its
// columns in that order and the epilogue writes them back in place.
struct BitScale {
  uint32_t m1, m2;  // bf16x2 multipliers: 2^(120+e), or 2^127 then 2^(e-7)
  bool two;
};
__device__ __forceinline__ BitScale bit_scale(float scale) {
  const uint32_t eb = (__float_as_uint(scale) >> 23) & 0xffu;  // e + 127
  BitScale d;
  if (eb <= 134u) {
    const uint32_t h = (eb + 120u) << 7;
    d.m1 = h | (h << 16);
    d.m2 = 0u;
    d.two = false;
  } else {
    const uint32_t h1 = 254u << 7, h2 = (eb - 7u) << 7;
    d.m1 = h1 | (h1 << 16);
    d.m2 = h2 | (h2 << 16);
    d.two = true;
  }
  return d;
}
// Four codes (lanes 0-3, byte i = lane i) -> bf16 pairs (lane 0, lane 2) and
// (lane 1, lane 3), times the block scale.
__device__ __forceinline__ void dequant4_bits(uint32_t w, const BitScale& d, uint32_t& even, uint32_t& odd) {
  uint32_t e = ((w << 8) & 0x80008000u) | ((w << 4) & 0x07f007f0u);
  uint32_t o = (w & 0x80008000u) | ((w >> 4) & 0x07f007f0u);
  e = mul_bf16x2(e, d.m1);
  o = mul_bf16x2(o, d.m1);
  if (d.two) {
    e = mul_bf16x2(e, d.m2);
    o = mul_bf16x2(o, d.m2);
  }
  even = e;
  odd = o;
}

__device__ __forceinline__ void set_abort(volatile int* abort_flag, uint32_t* status) {
  *abort_flag = 1;
  set_status(status, RKV_ERR_CUDA);
}

// Named-barrier reductions that keep a role's branches uniform after bounded
// waits: id 1 over the 128 softmax threads, id 2 over the 256 loaders.
__device__ __forceinline__ bool bar_all(int id, int n, bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)ok), "r"(id), "r"(n)
      : "memory");
  return r != 0;
}
__global__ void __launch_bounds__(kThreads, 1) mla_decode_kernel(const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);  // 1024-byte aligned atoms
  const uint32_t sbase = smem_u32(smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qi = blockIdx.y, split = blockIdx.x;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kSmemBar + kAbort);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kSmemBar + kTmemSlot);
  uint64_t* masks = reinterpret_cast<uint64_t*>(smem + kSmemBar + kMask);
  int32_t* slots = reinterpret_cast<int32_t*>(smem + kSmemRows);
  const uint32_t bar = sbase + kSmemBar;

  const int seq = p.seq_of_query[qi];
  const int len = max(p.seq_lens[seq], 0);
  const int n_pages_seq = (len + kTile - 1) / kTile;
  int page0 = 0, n_tiles;
  if (p.idx) {
    n_tiles = (p.k + kTile - 1) / kTile;
  } else {
    const int pps = (n_pages_seq + p.n_splits - 1) / p.n_splits;
    page0 = split * pps;
    n_tiles = max(0, min(pps, n_pages_seq - page0));
  }

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(bar + kBarKFull + 8 * i, kLoaders);
      mbar_init(bar + kBarKEmpty + 8 * i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar + kBarSFull + 8 * i, 1);
      mbar_init(bar + kBarSFree + 8 * i, 128);
      mbar_init(bar + kBarDrain + 8 * i, 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(bar + kBarTabFull + 8 * i, 32);
      mbar_init(bar + kBarTabFree + 8 * i, kLoaders);
    }
    mbar_init(bar + kBarPFull, 128);
    mbar_init(bar + kBarPvDone, 1);
    mbar_init(bar + kBarQReady, 128);
    mbar_init(bar + kBarQLoad, 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kQkWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (warp < 4) {
    // Q into TMEM as the A operand of S = Q K^T: one bulk copy per head row
    // into shared memory (all 73 KB in flight at once), then head h into lane
    // (h % 16) + 32 (h / 16), bf16 pairs along columns 0-287.  Lanes 16-31
    // read the same addresses (broadcast) and write the same values into
    // lanes 16-31, which hold O: the first O update overwrites them.
    if (warp == 0) {
      if (lane == 0) mbar_expect_tx(bar + kBarQLoad, kHeads * kQRowBytes);
      __syncwarp();
      const uint8_t* qsrc = reinterpret_cast<const uint8_t*>(p.q + (int64_t)qi * kHeads * kQk);
      for (int h = lane; h < kHeads; h += 32)
        bulk_g2s(sbase + kSmemQ + q_row_off(h), qsrc + h * kQRowBytes, kQRowBytes, bar + kBarQLoad);
    }
    const int h = warp * 16 + (lane & 15);
    const uint8_t* qs = smem + kSmemQ + q_row_off(h);
    const uint32_t tl = tmem + ((uint32_t)(warp * 32) << 16);
    if (mbar_wait_copy(bar + kBarQLoad, 0)) {
#pragma unroll 1
      for (int c = 0; c < kQk / 64; ++c) {
        uint32_t v[32];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint4 u = *reinterpret_cast<const uint4*>(qs + 16 * (8 * c + i));
          if (c < kV / 64) {  // latent lanes in stored order (0, 2, 1, 3) per group of four
            v[4 * i] = __byte_perm(u.x, u.y, 0x5410);
            v[4 * i + 1] = __byte_perm(u.x, u.y, 0x7632);
            v[4 * i + 2] = __byte_perm(u.z, u.w, 0x5410);
            v[4 * i + 3] = __byte_perm(u.z, u.w, 0x7632);
          } else {
            v[4 * i] = u.x;
            v[4 * i + 1] = u.y;
            v[4 * i + 2] = u.z;
            v[4 * i + 3] = u.w;
          }
        }
        tmem_st32(tl + 32 * c, v);
      }
      tmem_wait_st();
    } else {
      set_abort(abort_flag, p.status);
    }
    tc_fence_before();
    mbar_arrive(bar + kBarQReady);
  }

  if (warp == kQkWarp || warp == kQkWarp + 1) {
    // ------------------------------------------------------ MMA issuers
    // Warp 12 issues S = Q K^T of every tile once its stage is loaded and its
    // S buffer was read; warp 13 issues O += P V once P is written.  Each
    // blocks only on its own inputs, and the tensor pipe interleaves the two
    // streams.  The whole warp walks the tiles and waits (every lane polls the
    // barrier, so the warp stays converged); one elected lane issues a tile's
    // MMAs back to back from descriptors made once per stage, each K step a
    // constant added to the start-address field.  Issued that way an M = 64 x
    // N = 64 x K = 16 MMA takes ~32 cycles of the tensor pipe, against ~110
    // when a lone lane computed every descriptor (measured on this B200).
    const bool qk = warp == kQkWarp;
    if (n_tiles > 0) {
      bool ok = true;
      if (qk) {
        ok = __all_sync(0xffffffffu, mbar_wait(bar + kBarQReady, 0, abort_flag));
        for (int j = 0; ok && j < n_tiles; ++j) {
          const int b = j & 1;
          const bool got = mbar_wait(bar + kBarKFull + 8 * (j % kStages), (j / kStages) & 1, abort_flag) &&
                           (j < 2 || mbar_wait(bar + kBarSFree + 8 * b, ((j >> 1) - 1) & 1, abort_flag));
          ok = __all_sync(0xffffffffu, got);
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            const uint64_t kd = sw128_desc(sbase + kSmemK0 + (j % kStages) * kOperandBytes, 16, kAtom);
            const uint32_t d = tmem + kColS + 64 * b;
#pragma unroll
            for (int s = 0; s < kQk / 16; ++s)
              mma_bf16_ta(d, tmem + 8 * s, kd + (uint64_t)(((s >> 2) * kColBytes + (s & 3) * 32) >> 4), kIdescQK,
                          s > 0);
            mma_commit(bar + kBarSFull + 8 * b);
          }
          __syncwarp();
        }
      } else {
        const uint64_t pd = sw128_desc(sbase + kSmemP, 16, kAtom);
        for (int j = 0; ok && j < n_tiles; ++j) {
          ok = __all_sync(0xffffffffu, mbar_wait(bar + kBarPFull, j & 1, abort_flag));
          if (!ok) break;
          tc_fence_after();
          if (elect_one()) {
            const int b = j % kStages;
            const uint64_t vd = sw128_desc(sbase + kSmemK0 + b * kOperandBytes, kColBytes, kAtom);
#pragma unroll
            for (int qq = 0; qq < kTile / 16; ++qq) {
#pragma unroll
              for (int hf = 0; hf < 2; ++hf)
                mma_bf16(tmem + kLaneO + hf * 256, pd + (uint64_t)((qq * 32) >> 4),
                         vd + (uint64_t)((hf * 4 * kColBytes + qq * 2 * kAtom) >> 4), kIdescPV,
                         (j > 0 || qq > 0) ? 1u : 0u);
            }
            mma_commit(bar + kBarKEmpty + 8 * b);
            mma_commit(bar + kBarPvDone);
          }
          __syncwarp();
        }
      }
      if (elect_one()) {
        if (!ok) set_abort(abort_flag, p.status);
        const uint32_t drain = bar + kBarDrain + (qk ? 0 : 8);
        mma_commit(drain);  // every MMA issued here completes before the memory is freed
        const uint64_t t0 = now_ns();
        while (!mbar_test(drain, 0)) {
          if (now_ns() - t0 > kTimeoutNs) {
            set_abort(abort_flag, p.status);
            break;
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == kResolverWarp) {
    // ------------------------------------------------------------ resolver
    // Runs up to four tiles ahead of the loaders: lane l resolves rows l and
    // l + 32 of tile j to slots (page * 64 + row in page, -1 = no key) in
    // table j & 3 and the key mask j & 15.  Index loads for tile j + 1 are
    // issued before tile j's page-table loads are consumed.
    const int32_t* pt_row = p.page_table + (int64_t)seq * p.pt_stride;
    // The key position of row (j, l) or -1; for an index list, the entry.
    auto position = [&](int j, int row) -> int {
      const int pos = j * kTile + row;
      if (p.idx) {
        if (pos >= p.k) return -1;
        const int tok = __ldg(p.idx + (int64_t)qi * p.k + pos);
        return (tok >= 0 && tok < len) ? tok : -1;
      }
      return page0 * kTile + pos < len ? page0 * kTile + pos : -1;
    };
    // Later zeros of an index list repeat the top-k fill value: only the
    // list's first 0 is a key.  Tiles are resolved in list order (rows 0-31,
    // then 32-63), so the first 0 met here is the list's first.
    bool zero_seen = false;
    int tok0 = n_tiles > 0 ? position(0, lane) : -1, tok1 = n_tiles > 0 ? position(0, lane + 32) : -1;
    for (int j = 0; j < n_tiles; ++j) {
      const int tb = j & 3;
      if (p.idx) {
        const unsigned z0 = __ballot_sync(0xffffffffu, tok0 == 0), z1 = __ballot_sync(0xffffffffu, tok1 == 0);
        const unsigned keep0 = zero_seen ? 0u : (z0 & (0u - z0));
        const unsigned keep1 = (zero_seen || z0) ? 0u : (z1 & (0u - z1));
        zero_seen = zero_seen || (z0 | z1) != 0u;
        if (tok0 == 0 && !((keep0 >> lane) & 1u)) tok0 = -1;
        if (tok1 == 0 && !((keep1 >> lane) & 1u)) tok1 = -1;
      }
      const int pg0 = tok0 >= 0 ? __ldg(pt_row + tok0 / 64) : -1;
      const int pg1 = tok1 >= 0 ? __ldg(pt_row + tok1 / 64) : -1;
      const int ntok0 = j + 1 < n_tiles ? position(j + 1, lane) : -1;
      const int ntok1 = j + 1 < n_tiles ? position(j + 1, lane + 32) : -1;
      if (!__all_sync(0xffffffffu, j < 4 || mbar_wait(bar + kBarTabFree + 8 * tb, ((j >> 2) - 1) & 1, abort_flag))) {
        set_abort(abort_flag, p.status);
        break;
      }
      int s0 = -1, s1 = -1;
      if (tok0 >= 0) {
        if (pg0 >= 0 && pg0 < p.pool.n_pages) s0 = pg0 * 64 + (tok0 & 63);
        else set_status(p.status, RKV_ERR_INDEX_OUT_OF_RANGE);
      }
      if (tok1 >= 0) {
        if (pg1 >= 0 && pg1 < p.pool.n_pages) s1 = pg1 * 64 + (tok1 & 63);
        else set_status(p.status, RKV_ERR_INDEX_OUT_OF_RANGE);
      }
      slots[tb * 64 + lane] = s0;
      slots[tb * 64 + lane + 32] = s1;
      // dense: the tile is one page, 43 KB contiguous -- pull it into L2 now,
      // up to four tiles before the loaders read it
      if (!p.idx && lane == 0 && s0 >= 0)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(page_base(p.pool, p.layer, s0 >> 6)),
                     "r"((uint32_t)kPageBytes)
                     : "memory");
      const unsigned b0 = __ballot_sync(0xffffffffu, s0 >= 0), b1 = __ballot_sync(0xffffffffu, s1 >= 0);
      if (lane == 0) masks[j & 15] = ((uint64_t)b1 << 32) | b0;
      mbar_arrive(bar + kBarTabFull + 8 * tb);
      tok0 = ntok0;
      tok1 = ntok1;
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------- loaders
    // 256 threads per tile: lane (r8 = lane / 4, q = lane % 4) of loader warp
    // lw takes row 8 lw + r8: codes [128 s + 32 q, +32) for s = 0..3, the
    // row's 8 scales and RoPE bytes [32 q, +32), all as 256-bit loads.  The
    // loads of tile j + 1 are issued before tile j is stored.  Every wait is
    // per thread: a loader never waits for another loader.
    const int lt = tid - 128, lw = lt >> 5;
    const int r = 8 * lw + (lane >> 2);
    struct TileRegs {
      uint32_t codes[4][8], scl[8], rope[8];
    };
    auto load = [&](int j, TileRegs& t) -> bool {
      const int tb = j & 3;
      if (!mbar_wait(bar + kBarTabFull + 8 * tb, (j >> 2) & 1, abort_flag)) return false;
      const int slot = slots[tb * 64 + r];
      mbar_arrive(bar + kBarTabFree + 8 * tb);
      if (slot >= 0) {
        const uint8_t* pg = page_base(p.pool, p.layer, slot >> 6);
        const int off = slot & 63;
#pragma unroll
        for (int sg = 0; sg < 4; ++sg) ld_stream32(pg + codes_off(off) + sg * 128 + (lane & 3) * 32, t.codes[sg]);
        ld_cached32(pg + scales_off(off), t.scl);
        ld_stream32(pg + rope_off(off) + (lane & 3) * 32, t.rope);
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
#pragma unroll
          for (int sg = 0; sg < 4; ++sg) t.codes[sg][i] = 0u;
          t.scl[i] = 0x3f800000u;
          t.rope[i] = 0u;
        }
      }
      return true;
    };
    // Waits for the stage (the O update three tiles back; for tile 2, Q's
    // move out of the staging area), then dequantises.  Per store instruction the warp writes
    // 8 rows x 4 lanes of 16 B whose swizzled positions cover the 8 bank
    // groups evenly (4 wavefronts for 512 B, the minimum).
    auto store = [&](int j, const TileRegs& t) -> bool {
      const int b = j % kStages;
      if (j >= kStages && !mbar_wait(bar + kBarKEmpty + 8 * b, (j / kStages - 1) & 1, abort_flag)) return false;
      if (j == kStages - 1 && !mbar_wait(bar + kBarQReady, 0, abort_flag)) return false;  // Q staging read
      uint8_t* stage = smem + kSmemK0 + b * kOperandBytes;
#pragma unroll
      for (int sg = 0; sg < 4; ++sg) {
        const BitScale ds = bit_scale(__uint_as_float((lane & 2) ? t.scl[2 * sg + 1] : t.scl[2 * sg]));
        const int c0 = 8 * (2 * sg + ((lane & 3) >> 1)) + 4 * (lane & 1);
        uint32_t v[16];  // lanes in stored order, two per word
#pragma unroll
        for (int i = 0; i < 8; ++i) dequant4_bits(t.codes[sg][i], ds, v[2 * i], v[2 * i + 1]);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          *reinterpret_cast<uint4*>(stage + sw_off(r, c0 + k)) =
              make_uint4(v[4 * k], v[4 * k + 1], v[4 * k + 2], v[4 * k + 3]);
      }
      *reinterpret_cast<uint4*>(stage + sw_off(r, 64 + 2 * (lane & 3))) =
          make_uint4(t.rope[0], t.rope[1], t.rope[2], t.rope[3]);
      *reinterpret_cast<uint4*>(stage + sw_off(r, 64 + 2 * (lane & 3) + 1)) =
          make_uint4(t.rope[4], t.rope[5], t.rope[6], t.rope[7]);
      fence_proxy_async();
      mbar_arrive(bar + kBarKFull + 8 * b);
      return true;
    };
    TileRegs ta, tb;
    bool ok = n_tiles == 0 || load(0, ta);
    for (int j = 0; ok && j < n_tiles; j += 2) {
      if (j + 1 < n_tiles) ok = load(j + 1, tb);  // tile j is in ta
      ok = ok && store(j, ta);
      if (ok && j + 1 < n_tiles) {
        if (j + 2 < n_tiles) ok = load(j + 2, ta);  // tile j + 1 is in tb
        ok = ok && store(j + 1, tb);
      }
    }
    if (!ok) set_abort(abort_flag, p.status);
  } else {
    // ------------------------------------------------------------- softmax
    // Thread t of warp w handles heads hA = 16 w + t / 4 and hB = hA + 8 and,
    // of each 64-key tile, keys 8 r + 2 (t % 4) + {0, 1} for r = 0..7 (16-lane
    // TMEM accesses spread the 16 S rows over all 32 threads); the four threads
    // of a head pair combine maxima with shuffles.  The same accesses at lane
    // 16 reach O of the same two heads.
    const int g4 = lane >> 2, t4 = lane & 3;
    const int hA = warp * 16 + g4, hB = hA + 8;
    const uint32_t tS = tmem + ((uint32_t)(warp * 32) << 16), tO = tS + kLaneO;
    float mA = -INFINITY, mB = -INFINITY, lA = 0.0f, lB = 0.0f;  // m: per head; l: this thread's keys
    const unsigned long long sc2 = pk2(__float_as_uint(p.scale_log2), __float_as_uint(p.scale_log2));
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int b = j & 1;
      const bool got = mbar_wait(bar + kBarKFull + 8 * (j % kStages), (j / kStages) & 1, abort_flag) &&
                       mbar_wait(bar + kBarSFull + 8 * b, (j >> 1) & 1, abort_flag);
      if (!bar_all(1, 128, got)) {  // uniform over the four warps: TMEM accesses and barriers follow
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[32];  // register 4 r + k: head k < 2 ? hA : hB, key 8 r + 2 t4 + (k & 1)
      tmem_ld16x256x8(tS + kColS + 64 * b, sv);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(bar + kBarSFree + 8 * b);  // S buffer b may be overwritten
      const uint64_t mask = masks[j & 15];
      // Every key of the tile present (the same for all threads; all but the
      // last tile of a dense range): packed scaling, three-input maxima and
      // packed exponent arguments, with no masking.
      const bool full = mask == ~0ull;
      float mxA = -INFINITY, mxB = -INFINITY;
      if (full) {
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const unsigned long long x2 = mul_f32x2(pk2(sv[i], sv[i + 1]), sc2);
          sv[i] = (uint32_t)x2;
          sv[i + 1] = (uint32_t)(x2 >> 32);
        }
        mxA = fmaxf(__uint_as_float(sv[0]), __uint_as_float(sv[1]));
        mxB = fmaxf(__uint_as_float(sv[2]), __uint_as_float(sv[3]));
#pragma unroll
        for (int r = 1; r < 8; ++r) {
          mxA = fmax3(mxA, __uint_as_float(sv[4 * r]), __uint_as_float(sv[4 * r + 1]));
          mxB = fmax3(mxB, __uint_as_float(sv[4 * r + 2]), __uint_as_float(sv[4 * r + 3]));
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int key = 8 * (i >> 2) + 2 * t4 + (i & 1);
          const float x = ((mask >> key) & 1) ? __uint_as_float(sv[i]) * p.scale_log2 : -INFINITY;
          sv[i] = __float_as_uint(x);
          if (i & 2) mxB = fmaxf(mxB, x);
          else mxA = fmaxf(mxA, x);
        }
      }
      mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 1));
      mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, 2));
      mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 1));
      mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, 2));
      float alA = 1.0f, alB = 1.0f;
      bool rescale = false;
      if (mxA > -INFINITY && (mA == -INFINITY || mxA > mA + kRescaleLog2)) {
        alA = mA == -INFINITY ? 0.0f : ex2(mA - mxA);
        rescale |= mA != -INFINITY;
        mA = mxA;
        lA *= alA;
      }
      if (mxB > -INFINITY && (mB == -INFINITY || mxB > mB + kRescaleLog2)) {
        alB = mB == -INFINITY ? 0.0f : ex2(mB - mxB);
        rescale |= mB != -INFINITY;
        mB = mxB;
        lB *= alB;
      }
      uint32_t pa[8], pb[8];  // bf16 pairs: keys 8 r + 2 t4, +1 of hA / hB
      if (full) {  // mA and mB are finite here: the tile's maxima are
        const unsigned long long nA = pk2(__float_as_uint(-mA), __float_as_uint(-mA));
        const unsigned long long nB = pk2(__float_as_uint(-mB), __float_as_uint(-mB));
        unsigned long long sumA = 0ull, sumB = 0ull;  // the bf16-rounded weights, even and odd keys
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const unsigned long long a2 = add_f32x2(pk2(sv[4 * r], sv[4 * r + 1]), nA);
          const unsigned long long b2 = add_f32x2(pk2(sv[4 * r + 2], sv[4 * r + 3]), nB);
          pa[r] = pack_bf16x2(ex2(__uint_as_float((uint32_t)a2)), ex2(__uint_as_float((uint32_t)(a2 >> 32))));
          pb[r] = pack_bf16x2(ex2(__uint_as_float((uint32_t)b2)), ex2(__uint_as_float((uint32_t)(b2 >> 32))));
          sumA = add_f32x2(sumA, pk2(pa[r] << 16, pa[r] & 0xffff0000u));
          sumB = add_f32x2(sumB, pk2(pb[r] << 16, pb[r] & 0xffff0000u));
        }
        lA += __uint_as_float((uint32_t)sumA) + __uint_as_float((uint32_t)(sumA >> 32));
        lB += __uint_as_float((uint32_t)sumB) + __uint_as_float((uint32_t)(sumB >> 32));
      } else {
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const float x0 = __uint_as_float(sv[4 * r]), x1 = __uint_as_float(sv[4 * r + 1]);
          const float y0 = __uint_as_float(sv[4 * r + 2]), y1 = __uint_as_float(sv[4 * r + 3]);
          pa[r] = pack_bf16x2(x0 > -INFINITY ? ex2(x0 - mA) : 0.0f, x1 > -INFINITY ? ex2(x1 - mA) : 0.0f);
          pb[r] = pack_bf16x2(y0 > -INFINITY ? ex2(y0 - mB) : 0.0f, y1 > -INFINITY ? ex2(y1 - mB) : 0.0f);
          lA += __uint_as_float(pa[r] << 16) + __uint_as_float(pa[r] & 0xffff0000u);
          lB += __uint_as_float(pb[r] << 16) + __uint_as_float(pb[r] & 0xffff0000u);
        }
      }
      // P and O are free once the O update of tile j - 1 is done.
      if (!bar_all(1, 128, j == 0 || mbar_wait(bar + kBarPvDone, (j - 1) & 1, abort_flag))) {
        ok = false;
        break;
      }
      tc_fence_after();
      if (__any_sync(0xffffffffu, rescale)) {
        // O of hA / hB in lanes 16-31; 16-lane accesses leave Q and S alone.
#pragma unroll 1
        for (int c = 0; c < kV; c += 32) {
          uint32_t o[16];
          tmem_ld16x256(tO + c, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * ((i & 2) ? alB : alA));
          tmem_st16x256(tO + c, o);
        }
        tmem_wait_st();
      }
      uint8_t* prow = smem + kSmemP;
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        *reinterpret_cast<uint32_t*>(prow + sw_off(hA, r) + 4 * t4) = pa[r];
        *reinterpret_cast<uint32_t*>(prow + sw_off(hB, r) + 4 * t4) = pb[r];
      }
      fence_proxy_async();
      tc_fence_before();
      mbar_arrive(bar + kBarPFull);
    }
    if (ok && n_tiles > 0 && !bar_all(1, 128, mbar_wait(bar + kBarPvDone, (n_tiles - 1) & 1, abort_flag))) ok = false;
    if (!ok) set_abort(abort_flag, p.status);
    tc_fence_after();
    // Epilogue: the denominators sum the four threads' keys of each head.
    lA += __shfl_xor_sync(0xffffffffu, lA, 1);
    lA += __shfl_xor_sync(0xffffffffu, lA, 2);
    lB += __shfl_xor_sync(0xffffffffu, lB, 1);
    lB += __shfl_xor_sync(0xffffffffu, lB, 2);
    float scA = 0.0f, scB = 0.0f;
    float *dA, *dB;
    if (p.n_splits > 1) {
      const int64_t sA = ((int64_t)qi * p.n_splits + split) * kHeads + hA, sB = sA + 8;
      dA = p.ws_o + sA * kV;
      dB = p.ws_o + sB * kV;
      if (t4 == 0) {
        p.ws_ml[2 * sA] = mA;
        p.ws_ml[2 * sA + 1] = lA;
        p.ws_ml[2 * sB] = mB;
        p.ws_ml[2 * sB + 1] = lB;
      }
      scA = scB = 1.0f;
    } else {
      dA = p.out + ((int64_t)qi * kHeads + hA) * kV;
      dB = p.out + ((int64_t)qi * kHeads + hB) * kV;
      auto scale_of = [&](int h, float m, float l) {
        const float sink = p.sinks ? p.sinks[h] * 1.4426950408889634f : -INFINITY;
        const float M = fmaxf(m, sink);
        float sc = 0.0f;
        if (M > -INFINITY && M < INFINITY) {
          const float wo = m > -INFINITY ? ex2(m - M) : 0.0f;
          const float den = l * wo + (sink > -INFINITY ? ex2(sink - M) : 0.0f);
          if (den > 0.0f && den < INFINITY) sc = wo / den;
        }
        return sc;
      };
      scA = scale_of(hA, mA, lA);
      scB = scale_of(hB, mB, lB);
    }
    const bool have_o = ok && n_tiles > 0;
#pragma unroll 1
    for (int c = 0; c < kV; c += 64) {
      uint32_t o[32];
      if (have_o) {
        tmem_ld16x256x8(tO + c, o);
        tmem_wait_ld();
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        // stored columns 8 r + 2 t4 + {0, 1} are latent lanes l and l + 2
        const int col = c + 8 * r + 4 * (t4 >> 1) + (t4 & 1);
        float2 va = make_float2(0.f, 0.f), vb = make_float2(0.f, 0.f);
        if (have_o) {
          va = make_float2(__uint_as_float(o[4 * r]) * scA, __uint_as_float(o[4 * r + 1]) * scA);
          vb = make_float2(__uint_as_float(o[4 * r + 2]) * scB, __uint_as_float(o[4 * r + 3]) * scB);
        }
        dA[col] = va.x;
        dA[col + 2] = va.y;
        dB[col] = vb.x;
        dB[col + 2] = vb.y;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kQkWarp)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// Merges the split partials: per (query, head) the splits' (m, l, O) with the
// sink, as one softmax (the same guards as the single-split epilogue).
__global__ void __launch_bounds__(128) mla_combine_kernel(const float* __restrict__ ws_o,
                                                          const float* __restrict__ ws_ml, int n_splits,
                                                          const float* __restrict__ sinks, float* __restrict__ out) {
  const int qi = blockIdx.y, h = blockIdx.x;
  const float sink = sinks ? sinks[h] * 1.4426950408889634f : -INFINITY;
  float M = sink;
  for (int s = 0; s < n_splits; ++s) M = fmaxf(M, ws_ml[2 * (((int64_t)qi * n_splits + s) * kHeads + h)]);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float den = 0.0f;
  if (M > -INFINITY && M < INFINITY) {
    den = sink > -INFINITY ? ex2(sink - M) : 0.0f;
    for (int s = 0; s < n_splits; ++s) {
      const int64_t slot = ((int64_t)qi * n_splits + s) * kHeads + h;
      const float m = ws_ml[2 * slot];
      if (!(m > -INFINITY)) continue;
      const float w = ex2(m - M);
      den += w * ws_ml[2 * slot + 1];
      const float4 v = reinterpret_cast<const float4*>(ws_o + slot * kV)[threadIdx.x];
      acc.x += w * v.x;
      acc.y += w * v.y;
      acc.z += w * v.z;
      acc.w += w * v.w;
    }
  }
  const float inv = (den > 0.0f && den < INFINITY) ? 1.0f / den : 0.0f;
  reinterpret_cast<float4*>(out + ((int64_t)qi * kHeads + h) * kV)[threadIdx.x] =
      make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
}

}  // namespace mla
}  // namespace rkv

extern "C" int64_t rkv_mla_decode_workspace_bytes(int32_t n_q, int32_t n_splits) {
  if (n_q < 0 || n_splits < 1) return -1;
  if (n_splits == 1) return 0;
  return (int64_t)n_q * n_splits * rkv::mla::kHeads * (rkv::mla::kV + 2) * 4;
}

extern "C" rkv_status rkv_mla_decode_fp8(const rkv_pool_view* pool, int32_t layer, const int32_t* page_table,
                                         int64_t pt_stride, const int32_t* seq_lens, const int32_t* seq_of_query,
                                         const uint16_t* q, int32_t n_q, const int32_t* idx, int32_t k,
                                         const float* sinks, float softmax_scale, int32_t n_splits, void* workspace,
                                         float* out, uint32_t* d_status, rkv_stream_t stream) {
  using namespace rkv;
  using namespace rkv::mla;
  rkv_status st = check_pool(pool, "rkv_mla_decode_fp8");
  if (st != RKV_OK) return st;
  if (layer < 0 || layer >= pool->n_layers)
    return fail_layer(layer, pool->n_layers, "rkv_mla_decode_fp8: layer %d outside pool of %d layers", layer,
                      pool->n_layers);
  if (n_q < 0 || n_splits < 1 || n_splits > 65535 || pt_stride < 1 || (idx && (k < 0 || n_splits != 1)))
    return fail(RKV_ERR_SHAPE_MISMATCH, "rkv_mla_decode_fp8: n_q >= 0, pt_stride >= 1, 1 <= n_splits <= 65535 "
                "(1 with an index list) and k >= 0 are required");
  if (n_q == 0) {
    clear_error();
    return RKV_OK;
  }
  if (n_q > 65535) return fail_shape("n_q", 65535, n_q, "rkv_mla_decode_fp8: at most 65535 queries per call");
  if (!page_table || !seq_lens || !seq_of_query || !q || !aligned(q, 16) || !out || !aligned(out, 16) ||
      (n_splits > 1 && (!workspace || !aligned(workspace, 16))) || (idx && k > 0 && !aligned(idx, 4)))
    return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_mla_decode_fp8: page_table, seq_lens, seq_of_query, q (16-byte "
                "aligned), out (16-byte aligned) and, with n_splits > 1, workspace are required");
  if (!std::isfinite(softmax_scale))
    return fail(RKV_ERR_INVALID_ARGUMENT, "rkv_mla_decode_fp8: softmax_scale must be finite");
  // the shared-memory opt-in is per device
  static std::atomic<bool> attr_set[kMaxDevicesCached];
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevicesCached || !attr_set[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(mla_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemAlloc);
    if (e != cudaSuccess) return fail(RKV_ERR_CUDA, "rkv_mla_decode_fp8: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < kMaxDevicesCached) attr_set[dev].store(true, std::memory_order_release);
  }
  Params prm;
  prm.pool = *pool;
  prm.layer = layer;
  prm.page_table = page_table;
  prm.pt_stride = pt_stride;
  prm.seq_lens = seq_lens;
  prm.seq_of_query = seq_of_query;
  prm.q = q;
  prm.idx = idx;
  prm.k = idx ? k : 0;
  prm.sinks = sinks;
  prm.scale_log2 = (float)((double)softmax_scale * 1.4426950408889634);
  prm.n_splits = n_splits;
  float* ws = static_cast<float*>(workspace);
  prm.ws_o = ws;
  prm.ws_ml = ws ? ws + (int64_t)n_q * n_splits * kHeads * kV : nullptr;
  prm.out = out;
  prm.status = d_status;
  cudaStream_t s = (cudaStream_t)stream;
  mla_decode_kernel<<<dim3(n_splits, n_q), kThreads, kSmemAlloc, s>>>(prm);
  if (n_splits > 1) mla_combine_kernel<<<dim3(kHeads, n_q), 128, 0, s>>>(prm.ws_o, prm.ws_ml, n_splits, sinks, out);
  return check_launch("rkv_mla_decode_fp8");
}
