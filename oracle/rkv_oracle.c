/*
 * rkv_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C restatement, on the CPU, of rsLLM's KV-cache hot path.  It is the
 * checker the parity tests compare the CUDA path against, and the CPU
 * baseline that bench.py times beside the GPU.  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / reference legs load
 * it; the product library (rsllm_b200) never links, loads or calls it.
 *
 * What it restates (paths are relative to the rsLLM source tree):
 *   - FP8 E4M3FN KV codec:  crates/rsllm-backend-cpu/src/ops/dsv4_quant.rs
 *       e4m3fn_value :103-111 (table :71-78, subnormal step :82),
 *       e4m3fn_dequant :128-163, fp8_kv_quantize_row_inplace :316-362,
 *       libm_ldexpf :422-433, constants :43-66.
 *   - byte-level E4M3 codec: crates/rsllm-gguf/src/dequant/fp8_e4m3.rs:37-136.
 *   - top-k selection rule:  crates/rsllm-kvcache/src/dsv4/indexer.rs:218-236.
 *   - row append / chronological read semantics: crates/rsllm-kvcache/src/
 *       dsv4/swa.rs:73-94,131-149 and compressed.rs:203-205, generalised to a
 *       page-table-indexed pool (the reference has no paged pool; its plan is
 *       docs/03-HLD.md:363-369).
 *   - sparse row read: crates/rsllm-models/src/dsv4/attention.rs:549-560.
 *   - compressor emission: crates/rsllm-kvcache/src/dsv4/compressed.rs
 *       accumulate_wide :310-343, maybe_emit :360-417, finish_prefill_state
 *       :443-455, per_dim_softmax_aggregate :481-554; crates/rsllm-models/src/
 *       dsv4/compressor.rs:264-357 (APE bias, RMSNorm with an f64 sum of
 *       squares, RoPE at pos + 1 - ratio, quantize) with compress_rope_params
 *       :372-397; crates/rsllm-backend-cpu/src/ops/rope.rs:28-172 (YaRN).
 *       exp, log, pow, cos and sin are the host libm's, as in the reference.
 *   - indexer scoring: crates/rsllm-kvcache/src/dsv4/indexer.rs:198-216
 *       (ReLU of per-head dots, weighted sum), scale_factor :scale.
 *
 * Parity pin: the reference is Rust and cannot be built here (no cargo or
 * rustc), so this restatement is pinned by the reference's own known-answer
 * tests, transcribed into tests/golden/kat_reference.json with a file:line per
 * case, plus exhaustive checks (every f32 in [0, 448] through the snap, every
 * bf16 block amax through the exponent rule).  The paged layout itself has no
 * reference implementation and is checked for self-consistency only.
 *
 * Build: oracle/Makefile (gcc -O2, no fast-math, no FP contraction).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* Status bits shared with the product (include/rsllm_kv_cuda.h): an
 * operation over many rows ORs (1 << code) for every row that failed. */
enum {
    RKVO_OK = 0,
    RKVO_SHAPE_MISMATCH = 1,
    RKVO_INDEX_OUT_OF_RANGE = 2,
    RKVO_INVALID_LAYER = 3,
    RKVO_POOL_FULL = 4,
    RKVO_NON_FINITE_INPUT = 5,
};

/* Paged layout: one page = 64 token rows of one layer, structure of arrays:
 * codes[64][512] u8 | scales[64][8] f32 | rope[64][64] bf16 = 43008 bytes. */
#define PAGE_TOKENS 64
#define LATENT 512
#define ROPE 64
#define ROW_DIM (LATENT + ROPE)
#define BLOCK 64
#define NBLK (LATENT / BLOCK)
#define CODES_BYTES (PAGE_TOKENS * LATENT)
#define SCALES_BYTES (PAGE_TOKENS * NBLK * 4)
#define ROPE_BYTES (PAGE_TOKENS * ROPE * 2)
#define PAGE_BYTES (CODES_BYTES + SCALES_BYTES + ROPE_BYTES)

int rkvo_page_bytes(void) { return PAGE_BYTES; }

/* ------------------------------------------------------------------------ */
/* bit helpers                                                              */
/* ------------------------------------------------------------------------ */
static inline float f_from_bits(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static inline uint32_t bits_of(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }
static inline float bf16_to_f32(uint16_t h) { return f_from_bits((uint32_t)h << 16); }

/* f32 -> bf16, round to nearest even (NaN kept quiet). */
uint16_t rkvo_f32_to_bf16(float f) {
    uint32_t b = bits_of(f);
    if ((b & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((b >> 16) | 0x40u);
    b += 0x7fffu + ((b >> 16) & 1u);
    return (uint16_t)(b >> 16);
}

/* ------------------------------------------------------------------------ */
/* dsv4_quant.rs: the E4M3 simulation the reference runs on KV rows          */
/* ------------------------------------------------------------------------ */

/* dsv4_quant.rs:43-66 */
#define FP8_KV_GROUP 64
#define FP8_E4M3_MAX 448.0f
#define FP8_KV_AMAX_FLOOR 1.0e-4f
#define FP8_E4M3_CODE_MAX 126

/* dsv4_quant.rs:71-78: 2^(exp-7) for the normal exponents; slot 0 unused. */
static const float E4M3FN_EXP_SCALE[16] = {
    0.0f, 0.015625f, 0.03125f, 0.0625f, 0.125f, 0.25f, 0.5f, 1.0f,
    2.0f, 4.0f,      8.0f,     16.0f,   32.0f, 64.0f, 128.0f, 256.0f};

/* dsv4_quant.rs:103-111 */
float rkvo_e4m3fn_value(uint32_t i) {
    uint32_t e = (i >> 3) & 0xfu;
    float mant = (float)(i & 7u);
    if (e == 0) return mant * 0.001953125f; /* :82 subnormal step 1/512 */
    return (1.0f + mant * 0.125f) * E4M3FN_EXP_SCALE[e];
}

/* The magnitude-index search of dsv4_quant.rs:128-163 on ax = min(|x|, 448):
 * binary search for the largest code with value <= ax, then the one-sided
 * even tie-break against the next code. */
static int snap_index(float ax) {
    int lo = 0, hi = FP8_E4M3_CODE_MAX;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (rkvo_e4m3fn_value((uint32_t)mid) <= ax) lo = mid;
        else hi = mid - 1;
    }
    int best = lo;
    if (best < FP8_E4M3_CODE_MAX) {
        float best_diff = fabsf(ax - rkvo_e4m3fn_value((uint32_t)best));
        float next_diff = fabsf(ax - rkvo_e4m3fn_value((uint32_t)(best + 1)));
        if (next_diff < best_diff ||
            (next_diff == best_diff && ((best + 1) & 1) == 0 && (best & 1) != 0))
            best += 1;
    }
    return best;
}

/* dsv4_quant.rs:128-163.  Rust's f32::min returns the non-NaN operand, as
 * fminf does. */
float rkvo_e4m3fn_dequant(float x) {
    float sign = x < 0.0f ? -1.0f : 1.0f;
    float ax = fminf(fabsf(x), FP8_E4M3_MAX);
    return sign * rkvo_e4m3fn_value((uint32_t)snap_index(ax));
}

/* The code byte the snap above stands for: sign from (x < 0) -- so -0.0 maps
 * to 0x00 -- and the magnitude index in the low 7 bits. */
uint8_t rkvo_e4m3fn_code(float x) {
    uint8_t s = x < 0.0f ? 0x80 : 0x00;
    return (uint8_t)(s | (uint8_t)snap_index(fminf(fabsf(x), FP8_E4M3_MAX)));
}

/* Codes for a contiguous range of f32 bit patterns (exhaustive checks). */
typedef struct { uint32_t first; uint64_t n; uint8_t* out; } snap_job;
static void* snap_range_worker(void* p) {
    snap_job* j = (snap_job*)p;
    for (uint64_t i = 0; i < j->n; ++i)
        j->out[i] = rkvo_e4m3fn_code(f_from_bits(j->first + (uint32_t)i));
    return NULL;
}
void rkvo_e4m3fn_code_range(uint32_t first_bits, uint64_t n, uint8_t* out, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pthread_t th[256];
    snap_job jobs[256];
    uint64_t per = (n + (uint64_t)n_threads - 1) / (uint64_t)n_threads;
    int started = 0;
    for (int t = 0; t < n_threads; ++t) {
        uint64_t b = per * (uint64_t)t;
        if (b >= n) break;
        uint64_t e = b + per < n ? b + per : n;
        jobs[t].first = first_bits + (uint32_t)b;
        jobs[t].n = e - b;
        jobs[t].out = out + b;
        pthread_create(&th[t], NULL, snap_range_worker, &jobs[t]);
        ++started;
    }
    for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
}

/* dsv4_quant.rs:422-433 */
float rkvo_libm_ldexpf(float x, int n) {
    if (n < -126) n = -126;
    if (n > 127) n = 127;
    return x * f_from_bits((uint32_t)(n + 127) << 23);
}

/* The scale exponent of dsv4_quant.rs:346-355 for one block amax, exactly as
 * the reference evaluates it: floor, divide by 448, glibc log2f, ceil. */
int rkvo_scale_exponent(float amax) {
    if (amax < FP8_KV_AMAX_FLOOR) amax = FP8_KV_AMAX_FLOOR;
    float l = ceilf(log2f(amax / FP8_E4M3_MAX));
    /* Rust `as i32` saturates and maps NaN to 0. */
    if (l != l) return 0;
    if (l >= 2147483647.0f) return 2147483647;
    if (l <= -2147483648.0f) return (-2147483647 - 1);
    return (int)l;
}

/* dsv4_quant.rs:316-362, the reference's in-place f32 round trip. */
int rkvo_fp8_kv_quantize_row_inplace(float* x, int64_t x_len, int64_t head_dim, int64_t n_rot) {
    if (x_len != head_dim) return RKVO_SHAPE_MISMATCH;
    if (n_rot > head_dim) return RKVO_SHAPE_MISMATCH;
    int64_t n_nope = head_dim - n_rot;
    if (n_nope <= 0 || n_nope % FP8_KV_GROUP != 0) return RKVO_SHAPE_MISMATCH;
    for (int64_t b = 0; b < n_nope; b += FP8_KV_GROUP) {
        float amax = 0.0f;
        for (int i = 0; i < FP8_KV_GROUP; ++i) {
            float v = x[b + i];
            if (!isfinite(v)) return RKVO_NON_FINITE_INPUT; /* earlier blocks stay modified, as in Rust */
            float av = fabsf(v);
            if (av > amax) amax = av;
        }
        int e = rkvo_scale_exponent(amax);
        float scale = rkvo_libm_ldexpf(1.0f, e);
        for (int i = 0; i < FP8_KV_GROUP; ++i) {
            float t = x[b + i] / scale;
            if (t < -FP8_E4M3_MAX) t = -FP8_E4M3_MAX; /* f32::clamp */
            if (t > FP8_E4M3_MAX) t = FP8_E4M3_MAX;
            x[b + i] = rkvo_e4m3fn_dequant(t) * scale;
        }
    }
    return RKVO_OK;
}

/* ------------------------------------------------------------------------ */
/* Stored form of one row: the same arithmetic as above, keeping the code    */
/* bytes and the power-of-two scale instead of the simulated f32 values.     */
/* ------------------------------------------------------------------------ */

/* One bf16 row [head_dim] -> codes[n_nope], scales[n_nope/64] (f32 2^e),
 * rope[n_rot] (bf16 passthrough).  A non-finite latent lane rejects the row
 * before anything is written. */
int rkvo_quantize_row_bf16(const uint16_t* row, int64_t head_dim, int64_t n_rot,
                           uint8_t* codes, float* scales, uint16_t* rope) {
    if (n_rot > head_dim) return RKVO_SHAPE_MISMATCH;
    int64_t n_nope = head_dim - n_rot;
    if (n_nope <= 0 || n_nope % FP8_KV_GROUP != 0) return RKVO_SHAPE_MISMATCH;
    for (int64_t i = 0; i < n_nope; ++i)
        if (!isfinite(bf16_to_f32(row[i]))) return RKVO_NON_FINITE_INPUT;
    for (int64_t b = 0; b < n_nope; b += FP8_KV_GROUP) {
        float amax = 0.0f;
        for (int i = 0; i < FP8_KV_GROUP; ++i) {
            float av = fabsf(bf16_to_f32(row[b + i]));
            if (av > amax) amax = av;
        }
        int e = rkvo_scale_exponent(amax);
        float scale = rkvo_libm_ldexpf(1.0f, e);
        scales[b / FP8_KV_GROUP] = scale;
        for (int i = 0; i < FP8_KV_GROUP; ++i) {
            float t = bf16_to_f32(row[b + i]) / scale;
            if (t < -FP8_E4M3_MAX) t = -FP8_E4M3_MAX;
            if (t > FP8_E4M3_MAX) t = FP8_E4M3_MAX;
            codes[b + i] = rkvo_e4m3fn_code(t);
        }
    }
    memcpy(rope, row + n_nope, (size_t)n_rot * 2);
    return RKVO_OK;
}

/* The same stored form for an f32 row (the reference's own row type): the
 * codes and scale of dsv4_quant.rs:346-361 for each latent block, and the
 * RoPE lanes rounded to bf16 (the stored row holds bf16 RoPE). */
int rkvo_quantize_row_f32(const float* row, int64_t head_dim, int64_t n_rot,
                          uint8_t* codes, float* scales, uint16_t* rope) {
    if (n_rot > head_dim) return RKVO_SHAPE_MISMATCH;
    int64_t n_nope = head_dim - n_rot;
    if (n_nope <= 0 || n_nope % FP8_KV_GROUP != 0) return RKVO_SHAPE_MISMATCH;
    for (int64_t i = 0; i < n_nope; ++i)
        if (!isfinite(row[i])) return RKVO_NON_FINITE_INPUT;
    for (int64_t b = 0; b < n_nope; b += FP8_KV_GROUP) {
        float amax = 0.0f;
        for (int i = 0; i < FP8_KV_GROUP; ++i) {
            float av = fabsf(row[b + i]);
            if (av > amax) amax = av;
        }
        int e = rkvo_scale_exponent(amax);
        float scale = rkvo_libm_ldexpf(1.0f, e);
        scales[b / FP8_KV_GROUP] = scale;
        for (int i = 0; i < FP8_KV_GROUP; ++i) {
            float t = row[b + i] / scale;
            if (t < -FP8_E4M3_MAX) t = -FP8_E4M3_MAX;
            if (t > FP8_E4M3_MAX) t = FP8_E4M3_MAX;
            codes[b + i] = rkvo_e4m3fn_code(t);
        }
    }
    for (int64_t i = 0; i < n_rot; ++i) rope[i] = rkvo_f32_to_bf16(row[n_nope + i]);
    return RKVO_OK;
}

/* Checks a threshold table (exponent of y = (b - 127) + (mantissa >= t[b]))
 * against ceilf(log2f(y)) for every normal y with biased exponent in
 * [eb_lo, eb_hi].  Returns the number of disagreeing y; the first one's bits
 * go to *first_bad. */
typedef struct { const uint32_t* t; int eb_lo, eb_hi; uint64_t bad; uint32_t first; } table_job;

static void* table_worker(void* p) {
    table_job* j = (table_job*)p;
    j->bad = 0;
    j->first = 0;
    for (int eb = j->eb_lo; eb <= j->eb_hi; ++eb) {
        for (uint32_t m = 0; m < 0x800000u; ++m) {
            uint32_t yb = ((uint32_t)eb << 23) | m;
            int want = (int)ceilf(log2f(f_from_bits(yb)));
            int got = eb - 127 + (m >= j->t[eb] ? 1 : 0);
            if (got != want) {
                if (j->bad++ == 0) j->first = yb;
            }
        }
    }
    return NULL;
}

uint64_t rkvo_threshold_mismatches(const uint32_t* table, int eb_lo, int eb_hi, int n_threads, uint32_t* first_bad) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    int n = eb_hi - eb_lo + 1;
    if (n <= 0) return 0;
    if (n_threads > n) n_threads = n;
    pthread_t th[256];
    table_job jobs[256];
    for (int t = 0; t < n_threads; ++t) {
        jobs[t] = (table_job){table, eb_lo + (int)((int64_t)n * t / n_threads),
                              eb_lo + (int)((int64_t)n * (t + 1) / n_threads) - 1, 0, 0};
        pthread_create(&th[t], NULL, table_worker, &jobs[t]);
    }
    uint64_t bad = 0;
    *first_bad = 0;
    for (int t = 0; t < n_threads; ++t) {
        pthread_join(th[t], NULL);
        if (jobs[t].bad && bad == 0) *first_bad = jobs[t].first;
        bad += jobs[t].bad;
    }
    return bad;
}

/* Stored row -> bf16 [n_nope + n_rot]: (sign * e4m3fn_value) * scale, the
 * product the reference forms at dsv4_quant.rs:359, rounded to bf16. */
void rkvo_dequant_row_bf16(const uint8_t* codes, const float* scales, const uint16_t* rope,
                           int64_t n_nope, int64_t n_rot, uint16_t* out) {
    for (int64_t j = 0; j < n_nope; ++j) {
        uint8_t c = codes[j];
        float sign = (c & 0x80) ? -1.0f : 1.0f;
        float v = (sign * rkvo_e4m3fn_value(c & 0x7fu)) * scales[j / FP8_KV_GROUP];
        out[j] = rkvo_f32_to_bf16(v);
    }
    memcpy(out + n_nope, rope, (size_t)n_rot * 2);
}

/* ------------------------------------------------------------------------ */
/* fp8_e4m3.rs:37-136, the byte-level codec (differs on -0.0: 0x80 here).   */
/* ------------------------------------------------------------------------ */
float rkvo_fp8_e4m3_to_f32(uint8_t byte) {
    uint8_t sign_bit = byte & 0x80;
    uint8_t e = (byte >> 3) & 0x0f;
    uint8_t m = byte & 0x07;
    float a;
    if (e == 0) {
        a = (float)m / 512.0f;
    } else if (e == 0x0f && m == 0x07) {
        return NAN;
    } else {
        float mant_f = 1.0f + (float)m / 8.0f;
        int ei = (int)e - 7;
        float sc = ei >= 0 ? (float)(1ull << ei) : 1.0f / (float)(1ull << -ei);
        a = mant_f * sc;
    }
    return sign_bit ? -a : a;
}

uint8_t rkvo_f32_to_fp8_e4m3(float value) {
    if (isnan(value)) return 0x7f;
    uint8_t sign_bit = signbit(value) ? 0x80 : 0x00;
    float a = fabsf(value);
    if (a >= 448.0f) return sign_bit | 0x7e;
    if (a == 0.0f) return sign_bit;
    int unbiased = (int)floorf(log2f(a));
    if (unbiased < -6) {
        float scaled = a * 512.0f;
        uint32_t m = (uint32_t)rintf(scaled); /* round_ties_even */
        if (m >= 8) return sign_bit | 0x08;
        return (uint8_t)(sign_bit | (m & 0x07));
    }
    int e = unbiased + 7;
    if (e < 1) e = 1;
    if (e > 15) e = 15;
    float exp_scale = unbiased >= 0 ? (float)(1ull << unbiased) : 1.0f / (float)(1ull << -unbiased);
    float mant_f = (a / exp_scale - 1.0f) * 8.0f;
    int m = (int)rintf(mant_f);
    if (m == 8) {
        m = 0;
        e = e + 1;
        if (e >= 0x0f) return sign_bit | 0x7e;
    }
    if (m < 0) m = 0;
    if (m > 7) m = 7;
    return (uint8_t)(sign_bit | (e << 3) | (m & 0x07));
}

/* ------------------------------------------------------------------------ */
/* indexer.rs:218-236, top-k selection                                       */
/* ------------------------------------------------------------------------ */

/* The reference's repeated best-scan: effective_k = min(k, n) picks, each the
 * not-yet-selected row with the largest score by strict `>` from -inf (ties go
 * to the lowest index; NaN and -inf never win).  When no candidate beats -inf
 * the pick is index 0, emitted again.  Returns the number of indices written. */
int64_t rkvo_select_top_k_scan(const float* scores, int64_t n, int64_t top_k, int32_t* out) {
    if (n <= 0 || top_k <= 0) return 0;
    int64_t k = top_k < n ? top_k : n;
    uint8_t* allowed = (uint8_t*)calloc((size_t)n, 1);
    for (int64_t it = 0; it < k; ++it) {
        int64_t best_idx = 0;
        float best_score = -INFINITY;
        for (int64_t c = 0; c < n; ++c) {
            if (!allowed[c] && scores[c] > best_score) {
                best_score = scores[c];
                best_idx = c;
            }
        }
        allowed[best_idx] = 1;
        out[it] = (int32_t)best_idx;
    }
    free(allowed);
    return k;
}

/* The same output computed by a sort: the candidates that can win (score >
 * -inf, not NaN) in descending score with ascending index on ties, then index
 * 0 repeated up to effective_k.  -0.0 and +0.0 compare equal under `>`, so
 * they are ordered as one value. */
static inline uint64_t topk_key(float s, int64_t idx) {
    if (s == 0.0f) s = 0.0f; /* fold -0.0 into +0.0 */
    uint32_t b = bits_of(s);
    uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((uint64_t)ord << 32) | (uint64_t)(0xffffffffu - (uint32_t)idx);
}
static int cmp_desc_u64(const void* a, const void* b) {
    uint64_t x = *(const uint64_t*)a, y = *(const uint64_t*)b;
    return x < y ? 1 : (x > y ? -1 : 0);
}
int64_t rkvo_select_top_k_sorted(const float* scores, int64_t n, int64_t top_k, int32_t* out) {
    if (n <= 0 || top_k <= 0) return 0;
    int64_t k = top_k < n ? top_k : n;
    uint64_t* keys = (uint64_t*)malloc((size_t)n * 8);
    int64_t m = 0;
    for (int64_t c = 0; c < n; ++c)
        if (scores[c] > -INFINITY) keys[m++] = topk_key(scores[c], c);
    qsort(keys, (size_t)m, 8, cmp_desc_u64);
    int64_t i = 0;
    for (; i < k && i < m; ++i) out[i] = (int32_t)(0xffffffffu - (uint32_t)(keys[i] & 0xffffffffu));
    for (; i < k; ++i) out[i] = 0;
    free(keys);
    return k;
}

/* Batched top-k over rows of a [n_q][ld] score matrix; query q sees keys
 * [0, n_visible[q]) (causal masking = the pool holding only visible rows).
 * Indices past a query's effective_k are -1. */
typedef struct {
    const float* scores; int64_t ld; int32_t q0, q1; const int32_t* n_visible;
    int32_t k; int32_t* out; int scan;
} topk_job;
static void* topk_worker(void* p) {
    topk_job* j = (topk_job*)p;
    for (int32_t q = j->q0; q < j->q1; ++q) {
        int32_t* o = j->out + (int64_t)q * j->k;
        int64_t got = j->scan ? rkvo_select_top_k_scan(j->scores + (int64_t)q * j->ld, j->n_visible[q], j->k, o)
                              : rkvo_select_top_k_sorted(j->scores + (int64_t)q * j->ld, j->n_visible[q], j->k, o);
        for (int64_t i = got; i < j->k; ++i) o[i] = -1;
    }
    return NULL;
}
void rkvo_topk_batch(const float* scores, int64_t ld, int32_t n_q, const int32_t* n_visible,
                     int32_t k, int32_t* out, int scan, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pthread_t th[256];
    topk_job jobs[256];
    int32_t per = (n_q + n_threads - 1) / n_threads;
    int started = 0;
    for (int t = 0; t < n_threads; ++t) {
        int32_t b = per * t;
        if (b >= n_q) break;
        jobs[t] = (topk_job){scores, ld, b, b + per < n_q ? b + per : n_q, n_visible, k, out, scan};
        pthread_create(&th[t], NULL, topk_worker, &jobs[t]);
        ++started;
    }
    for (int t = 0; t < started; ++t) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------------ */
/* Paged pool model                                                          */
/* ------------------------------------------------------------------------ */
/* Pool: n_layers regions of n_pages pages each; page p of layer l starts at
 * pool + (l * n_pages + p) * PAGE_BYTES.  A slot is page * 64 + offset. */
static inline uint8_t* page_ptr(uint8_t* pool, int64_t n_pages, int32_t layer, int64_t page) {
    return pool + ((int64_t)layer * n_pages + page) * (int64_t)PAGE_BYTES;
}

typedef struct {
    uint8_t* pool; int64_t n_pages; int32_t n_layers; int32_t layer0; int32_t n_layers_in;
    const void* rows; int is_f32; int64_t n_tokens; const int32_t* slots;
    int64_t r0, r1; uint32_t status;
} append_job;

static void* append_worker(void* p) {
    append_job* j = (append_job*)p;
    uint8_t codes[LATENT];
    float scales[NBLK];
    uint16_t rope[ROPE];
    for (int64_t r = j->r0; r < j->r1; ++r) {
        int64_t li = r / j->n_tokens, t = r % j->n_tokens;
        int32_t layer = j->layer0 + (int32_t)li;
        int32_t slot = j->slots[t];
        if (slot < 0) continue; /* padding row */
        if (layer < 0 || layer >= j->n_layers) { j->status |= 1u << RKVO_INVALID_LAYER; continue; }
        int64_t page = slot / PAGE_TOKENS, off = slot % PAGE_TOKENS;
        if (page >= j->n_pages) { j->status |= 1u << RKVO_INDEX_OUT_OF_RANGE; continue; }
        int rc = j->is_f32
                     ? rkvo_quantize_row_f32((const float*)j->rows + r * ROW_DIM, ROW_DIM, ROPE, codes, scales, rope)
                     : rkvo_quantize_row_bf16((const uint16_t*)j->rows + r * ROW_DIM, ROW_DIM, ROPE, codes, scales,
                                              rope);
        if (rc != RKVO_OK) { j->status |= 1u << rc; continue; }
        uint8_t* pg = page_ptr(j->pool, j->n_pages, layer, page);
        memcpy(pg + off * LATENT, codes, LATENT);
        memcpy(pg + CODES_BYTES + off * NBLK * 4, scales, NBLK * 4);
        memcpy(pg + CODES_BYTES + SCALES_BYTES + off * ROPE * 2, rope, ROPE * 2);
    }
    return NULL;
}

/* rows: [n_layers_in][n_tokens][576] bf16 (is_f32 = 0) or f32 (is_f32 = 1);
 * slots: [n_tokens] (shared by the layers, < 0 = skip).  Returns the OR of
 * (1 << status) over failed rows. */
uint32_t rkvo_append_rows(uint8_t* pool, int64_t n_pages, int32_t n_layers, int32_t layer0,
                          int32_t n_layers_in, const void* rows, int is_f32, int64_t n_tokens,
                          const int32_t* slots, int n_threads) {
    int64_t n_rows = (int64_t)n_layers_in * n_tokens;
    if (n_rows <= 0) return 0;
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pthread_t th[256];
    append_job jobs[256];
    int64_t per = (n_rows + n_threads - 1) / n_threads;
    int started = 0;
    for (int t = 0; t < n_threads; ++t) {
        int64_t b = per * t;
        if (b >= n_rows) break;
        jobs[t] = (append_job){pool, n_pages, n_layers, layer0, n_layers_in, rows, is_f32, n_tokens, slots,
                               b, b + per < n_rows ? b + per : n_rows, 0};
        if (n_threads == 1) append_worker(&jobs[t]);
        else pthread_create(&th[t], NULL, append_worker, &jobs[t]);
        ++started;
    }
    uint32_t st = 0;
    for (int t = 0; t < started; ++t) {
        if (n_threads > 1) pthread_join(th[t], NULL);
        st |= jobs[t].status;
    }
    return st;
}

/* Read one stored row (layer, page, off) back as bf16 [576]. */
static void read_row(const uint8_t* pool, int64_t n_pages, int32_t layer, int64_t page, int64_t off,
                     uint16_t* out) {
    const uint8_t* pg = page_ptr((uint8_t*)pool, n_pages, layer, page);
    rkvo_dequant_row_bf16(pg + off * LATENT, (const float*)(pg + CODES_BYTES + off * NBLK * 4),
                          (const uint16_t*)(pg + CODES_BYTES + SCALES_BYTES + off * ROPE * 2),
                          LATENT, ROPE, out);
}

typedef struct {
    const uint8_t* pool; int64_t n_pages; int32_t layer;
    const int32_t* page_table; int64_t pt_stride; const int32_t* cu_seqlens; int32_t n_seq;
    uint16_t* out; int64_t r0, r1; uint32_t status;
} gather_job;

static void* gather_worker(void* p) {
    gather_job* j = (gather_job*)p;
    int32_t s = 0;
    for (int64_t r = j->r0; r < j->r1; ++r) {
        while (s + 1 <= j->n_seq && j->cu_seqlens[s + 1] <= r) ++s;
        int64_t t = r - j->cu_seqlens[s];
        int32_t page = j->page_table[(int64_t)s * j->pt_stride + t / PAGE_TOKENS];
        if (page < 0 || page >= j->n_pages) {
            j->status |= 1u << RKVO_INDEX_OUT_OF_RANGE;
            memset(j->out + r * ROW_DIM, 0, ROW_DIM * 2);
            continue;
        }
        read_row(j->pool, j->n_pages, j->layer, page, t % PAGE_TOKENS, j->out + r * ROW_DIM);
    }
    return NULL;
}

/* Chronological read of n_seq sequences (swa.rs:131 rows() generalised to a
 * page table): row t of sequence s lands at out[cu_seqlens[s] + t]. */
uint32_t rkvo_gather_rows(const uint8_t* pool, int64_t n_pages, int32_t n_layers, int32_t layer,
                          const int32_t* page_table, int64_t pt_stride, const int32_t* cu_seqlens,
                          int32_t n_seq, uint16_t* out, int n_threads) {
    if (layer < 0 || layer >= n_layers) return 1u << RKVO_INVALID_LAYER;
    int64_t n_rows = cu_seqlens[n_seq];
    if (n_rows <= 0) return 0;
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pthread_t th[256];
    gather_job jobs[256];
    int64_t per = (n_rows + n_threads - 1) / n_threads;
    int started = 0;
    for (int t = 0; t < n_threads; ++t) {
        int64_t b = per * t;
        if (b >= n_rows) break;
        jobs[t] = (gather_job){pool, n_pages, layer, page_table, pt_stride, cu_seqlens, n_seq, out,
                               b, b + per < n_rows ? b + per : n_rows, 0};
        if (n_threads == 1) gather_worker(&jobs[t]);
        else pthread_create(&th[t], NULL, gather_worker, &jobs[t]);
        ++started;
    }
    uint32_t st = 0;
    for (int t = 0; t < started; ++t) {
        if (n_threads > 1) pthread_join(th[t], NULL);
        st |= jobs[t].status;
    }
    return st;
}

typedef struct {
    const uint8_t* pool; int64_t n_pages; int32_t layer;
    const int32_t* page_table; int64_t pt_stride; const int32_t* seq_of_query; const int32_t* seq_lens;
    const int32_t* idx; int32_t k; uint16_t* out; int64_t r0, r1; uint32_t status;
} sparse_job;

static void* sparse_worker(void* p) {
    sparse_job* j = (sparse_job*)p;
    for (int64_t r = j->r0; r < j->r1; ++r) {
        int64_t q = r / j->k;
        int32_t s = j->seq_of_query[q];
        int32_t t = j->idx[r];
        uint16_t* o = j->out + r * ROW_DIM;
        if (t < 0) { memset(o, 0, ROW_DIM * 2); continue; } /* unused selection slot */
        if (t >= j->seq_lens[s]) { j->status |= 1u << RKVO_INDEX_OUT_OF_RANGE; memset(o, 0, ROW_DIM * 2); continue; }
        int32_t page = j->page_table[(int64_t)s * j->pt_stride + t / PAGE_TOKENS];
        if (page < 0 || page >= j->n_pages) { j->status |= 1u << RKVO_INDEX_OUT_OF_RANGE; memset(o, 0, ROW_DIM * 2); continue; }
        read_row(j->pool, j->n_pages, j->layer, page, t % PAGE_TOKENS, o);
    }
    return NULL;
}

/* Selected-row read (attention.rs:549-560 reads only rows in the top-k set):
 * out[q][i] = row idx[q][i] of sequence seq_of_query[q]. */
uint32_t rkvo_sparse_gather_rows(const uint8_t* pool, int64_t n_pages, int32_t n_layers, int32_t layer,
                                 const int32_t* page_table, int64_t pt_stride, const int32_t* seq_of_query,
                                 const int32_t* seq_lens, const int32_t* idx, int32_t n_q, int32_t k,
                                 uint16_t* out, int n_threads) {
    if (layer < 0 || layer >= n_layers) return 1u << RKVO_INVALID_LAYER;
    int64_t n_rows = (int64_t)n_q * k;
    if (n_rows <= 0) return 0;
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pthread_t th[256];
    sparse_job jobs[256];
    int64_t per = (n_rows + n_threads - 1) / n_threads;
    int started = 0;
    for (int t = 0; t < n_threads; ++t) {
        int64_t b = per * t;
        if (b >= n_rows) break;
        jobs[t] = (sparse_job){pool, n_pages, layer, page_table, pt_stride, seq_of_query, seq_lens, idx, k, out,
                               b, b + per < n_rows ? b + per : n_rows, 0};
        if (n_threads == 1) sparse_worker(&jobs[t]);
        else pthread_create(&th[t], NULL, sparse_worker, &jobs[t]);
        ++started;
    }
    uint32_t st = 0;
    for (int t = 0; t < started; ++t) {
        if (n_threads > 1) pthread_join(th[t], NULL);
        st |= jobs[t].status;
    }
    return st;
}

/* Whole-page copies for copy-on-write and compaction, every layer. */
void rkvo_copy_pages(uint8_t* pool, int64_t n_pages, int32_t n_layers, const int32_t* src,
                     const int32_t* dst, int64_t n) {
    for (int32_t l = 0; l < n_layers; ++l)
        for (int64_t i = 0; i < n; ++i)
            memcpy(page_ptr(pool, n_pages, l, dst[i]), page_ptr(pool, n_pages, l, src[i]), PAGE_BYTES);
}

/* ------------------------------------------------------------------------ */
/* MLA decode attention over the paged pool                                  */
/* ------------------------------------------------------------------------ */
/* The mixed sweep of crates/rsllm-models/src/dsv4/attention.rs:493-663 for
 * one query position, restated over a sequence's pooled rows:
 *   keys    = every row [0, len) of the query's sequence (dense), or the rows
 *             whose positions appear in idx[q][0..k) and are < len (sparse:
 *             the `allowed` set of :548-556, duplicates count once);
 *   logit   = (sum_d q_h[d] * k[d]) * scale over the 576 stored lanes
 *             (dequantised latent + bf16 RoPE), rows in ascending order (:582-606);
 *   softmax = max over the sink and the logits, exp(l - max), the sink's
 *             exp(sink - max) in the denominator only (:627-643);
 *   output  = sum (e * inv_denom) * v over the 512 latent lanes (:646-663);
 *   a non-finite max or a zero / non-finite denominator gives zeros (:618-641).
 * q: bf16 [n_q][64][576]; out: f32 [n_q][64][512]; sinks: f32 [64] or NULL. */
#define MLA_HEADS 64
#define MLA_QK 576
#define MLA_V 512

typedef struct {
    const uint8_t* pool; int64_t n_pages; int32_t layer;
    const int32_t* pt; int64_t pt_stride; const int32_t* seq_lens; const int32_t* seq_of_query;
    const uint16_t* q; const int32_t* idx; int32_t k; const float* sinks; float scale; float* out;
    int32_t q0, q1; uint32_t status;
} mla_job;

static int mla_row(const mla_job* j, int32_t seq, int64_t pos, float* row) {
    int32_t page = j->pt[(int64_t)seq * j->pt_stride + pos / PAGE_TOKENS];
    if (page < 0 || page >= j->n_pages) return 0;
    const uint8_t* pg = page_ptr((uint8_t*)j->pool, j->n_pages, j->layer, page);
    int64_t off = pos % PAGE_TOKENS;
    const uint8_t* codes = pg + off * LATENT;
    const float* sc = (const float*)(pg + CODES_BYTES + off * NBLK * 4);
    const uint16_t* rope = (const uint16_t*)(pg + CODES_BYTES + SCALES_BYTES + off * ROPE * 2);
    for (int d = 0; d < LATENT; ++d) {
        uint8_t c = codes[d];
        float sign = (c & 0x80) ? -1.0f : 1.0f;
        row[d] = (sign * rkvo_e4m3fn_value(c & 0x7fu)) * sc[d / BLOCK];
    }
    for (int d = 0; d < ROPE; ++d) row[LATENT + d] = bf16_to_f32(rope[d]);
    return 1;
}

static void* mla_worker(void* p) {
    mla_job* j = (mla_job*)p;
    for (int32_t qi = j->q0; qi < j->q1; ++qi) {
        int32_t seq = j->seq_of_query[qi];
        int64_t len = j->seq_lens[seq];
        /* the key set in ascending row order */
        uint8_t* allowed = (uint8_t*)calloc((size_t)(len > 0 ? len : 1), 1);
        if (j->idx) {
            for (int32_t t = 0; t < j->k; ++t) {
                int32_t c = j->idx[(int64_t)qi * j->k + t];
                if (c >= 0 && c < len) allowed[c] = 1;
            }
        } else {
            memset(allowed, 1, (size_t)len);
        }
        int64_t n_keys = 0;
        for (int64_t c = 0; c < len; ++c) n_keys += allowed[c];
        float* rows = (float*)malloc((size_t)(n_keys > 0 ? n_keys : 1) * MLA_QK * sizeof(float));
        int64_t r = 0;
        for (int64_t c = 0; c < len; ++c) {
            if (!allowed[c]) continue;
            if (!mla_row(j, seq, c, rows + r * MLA_QK)) {
                j->status |= 1u << RKVO_INDEX_OUT_OF_RANGE; /* a row on a bad page is not a key */
                continue;
            }
            ++r;
        }
        n_keys = r;
        float* logits = (float*)malloc((size_t)(n_keys > 0 ? n_keys : 1) * sizeof(float));
        for (int h = 0; h < MLA_HEADS; ++h) {
            const uint16_t* qh = j->q + ((int64_t)qi * MLA_HEADS + h) * MLA_QK;
            float qf[MLA_QK];
            for (int d = 0; d < MLA_QK; ++d) qf[d] = bf16_to_f32(qh[d]);
            float sink = j->sinks ? j->sinks[h] : -INFINITY;
            float max_logit = sink;
            for (int64_t t = 0; t < n_keys; ++t) {
                const float* kr = rows + t * MLA_QK;
                float dot = 0.0f;
                for (int d = 0; d < MLA_QK; ++d) dot += qf[d] * kr[d];
                float l = dot * j->scale;
                if (l > max_logit) max_logit = l;
                logits[t] = l;
            }
            float* oh = j->out + ((int64_t)qi * MLA_HEADS + h) * MLA_V;
            for (int d = 0; d < MLA_V; ++d) oh[d] = 0.0f;
            if (!isfinite(max_logit)) continue;
            float denom = isfinite(sink) ? expf(sink - max_logit) : 0.0f;
            for (int64_t t = 0; t < n_keys; ++t) {
                logits[t] = expf(logits[t] - max_logit);
                denom += logits[t];
            }
            if (!isfinite(denom) || denom == 0.0f) continue;
            float inv = 1.0f / denom;
            for (int64_t t = 0; t < n_keys; ++t) {
                float w = logits[t] * inv;
                const float* vr = rows + t * MLA_QK;
                for (int d = 0; d < MLA_V; ++d) oh[d] += w * vr[d];
            }
        }
        free(logits);
        free(rows);
        free(allowed);
    }
    return NULL;
}

uint32_t rkvo_mla_decode(const uint8_t* pool, int64_t n_pages, int32_t n_layers, int32_t layer,
                         const int32_t* page_table, int64_t pt_stride, const int32_t* seq_lens,
                         const int32_t* seq_of_query, const uint16_t* q, int32_t n_q, const int32_t* idx,
                         int32_t k, const float* sinks, float scale, float* out, int n_threads) {
    if (n_q <= 0) return 0;
    if (layer < 0 || layer >= n_layers) return 1u << RKVO_INVALID_LAYER;
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    if (n_threads > n_q) n_threads = n_q;
    pthread_t th[256];
    mla_job jobs[256];
    for (int t = 0; t < n_threads; ++t) {
        jobs[t] = (mla_job){pool, n_pages, layer, page_table, pt_stride, seq_lens, seq_of_query, q, idx, k, sinks,
                            scale, out, (int32_t)((int64_t)n_q * t / n_threads),
                            (int32_t)((int64_t)n_q * (t + 1) / n_threads), 0};
        if (n_threads == 1) mla_worker(&jobs[t]);
        else pthread_create(&th[t], NULL, mla_worker, &jobs[t]);
    }
    uint32_t st = 0;
    for (int t = 0; t < n_threads; ++t) {
        if (n_threads > 1) pthread_join(th[t], NULL);
        st |= jobs[t].status;
    }
    return st;
}

/* ------------------------------------------------------------------------ */
/* Compressor emission: crates/rsllm-kvcache/src/dsv4/compressed.rs          */
/* (window state, per-dimension softmax aggregate) and                       */
/* crates/rsllm-models/src/dsv4/compressor.rs (APE bias, RMSNorm, RoPE,      */
/* quantize), with crates/rsllm-backend-cpu/src/ops/rope.rs for the rotation. */
/* ------------------------------------------------------------------------ */

/* compressed.rs:481-554.  coff 2: lane p = state[r][j] (lower half), lane c =
 * state[ratio + r][head_dim + j] (upper half), one softmax over both. */
void rkvo_per_dim_softmax_aggregate(const float* state_kv, const float* state_score, int64_t ratio,
                                    int64_t head_dim, int64_t coff, int64_t width, float* out) {
    for (int64_t j = 0; j < head_dim; ++j) {
        float max_s = -INFINITY;
        if (coff == 2) {
            for (int64_t r = 0; r < ratio; ++r) {
                float sp = state_score[r * width + j];
                float sc = state_score[(ratio + r) * width + head_dim + j];
                if (sp > max_s) max_s = sp;
                if (sc > max_s) max_s = sc;
            }
        } else {
            for (int64_t r = 0; r < ratio; ++r) {
                float s = state_score[r * width + j];
                if (s > max_s) max_s = s;
            }
        }
        if (max_s <= -INFINITY * 0.5f) { out[j] = 0.0f; continue; }
        float denom = 0.0f, numer = 0.0f;
        if (coff == 2) {
            for (int64_t r = 0; r < ratio; ++r) {
                int64_t off_p = r * width + j, off_c = (ratio + r) * width + head_dim + j;
                float wp = expf(state_score[off_p] - max_s);
                float wc = expf(state_score[off_c] - max_s);
                denom += wp + wc;
                numer += wp * state_kv[off_p] + wc * state_kv[off_c];
            }
        } else {
            for (int64_t r = 0; r < ratio; ++r) {
                int64_t off = r * width + j;
                float w = expf(state_score[off] - max_s);
                denom += w;
                numer += w * state_kv[off];
            }
        }
        out[j] = denom > 0.0f ? numer / denom : 0.0f;
    }
}

static inline int64_t cmp_coff(int64_t ratio) { return ratio == 4 ? 2 : 1; }

/* compressed.rs:310-343 (accumulate_wide) + :360-417 (maybe_emit) for a state
 * of [coff*ratio][coff*head_dim] kv and score rows.  Returns 1 when the
 * window is full and out[head_dim] holds the aggregate (the capacity check
 * of the reference's row store is the caller's). */
int rkvo_compressor_accumulate(float* state_kv, float* state_score, uint32_t* state_count, int64_t ratio,
                               int64_t head_dim, const float* kv, const float* score, float* out) {
    int64_t coff = cmp_coff(ratio), width = coff * head_dim, slot = *state_count;
    int64_t row = coff == 2 ? ratio + slot : slot;
    memcpy(state_kv + row * width, kv, (size_t)width * 4);
    memcpy(state_score + row * width, score, (size_t)width * 4);
    *state_count += 1;
    if (*state_count < (uint32_t)ratio) return 0;
    rkvo_per_dim_softmax_aggregate(state_kv, state_score, ratio, head_dim, coff, width, out);
    if (coff == 2) {
        for (int64_t r = 0; r < ratio; ++r) {
            memmove(state_kv + r * width, state_kv + (ratio + r) * width, (size_t)width * 4);
            memmove(state_score + r * width, state_score + (ratio + r) * width, (size_t)width * 4);
        }
        for (int64_t r = 0; r < ratio; ++r) {
            memmove(state_kv + (ratio + r) * width, state_kv + r * width, (size_t)width * 4);
            memmove(state_score + (ratio + r) * width, state_score + r * width, (size_t)width * 4);
        }
    } else {
        for (int64_t i = 0; i < ratio * width; ++i) { state_kv[i] = 0.0f; state_score[i] = -INFINITY; }
    }
    *state_count = 0;
    return 1;
}

/* compressed.rs:443-455. */
void rkvo_compressor_finish_prefill(float* state_kv, float* state_score, uint32_t* state_count, int64_t ratio,
                                    int64_t head_dim, int64_t n_tokens) {
    int64_t coff = cmp_coff(ratio), width = coff * head_dim, rem = n_tokens % ratio;
    for (int64_t row = coff == 2 ? ratio + rem : rem; row < coff * ratio; ++row)
        for (int64_t j = 0; j < width; ++j) { state_kv[row * width + j] = 0.0f; state_score[row * width + j] = -INFINITY; }
    *state_count = (uint32_t)rem;
}

/* rope.rs:28-31 */
static float yarn_ramp(float low, float high, int32_t i0) {
    float y = ((float)(i0 / 2) - low) / fmaxf(high - low, 0.001f);
    y = y < 0.0f ? 0.0f : (y > 1.0f ? 1.0f : y);
    return 1.0f - y;
}

/* rope.rs:37-39 (PI is f32 pi) */
static float yarn_corr_dim(int32_t n_dims, uint64_t n_ctx_orig, float n_rot, float base) {
    const float pi = 3.14159265358979323846f;
    return ((float)n_dims * logf((float)n_ctx_orig / (n_rot * 2.0f * pi))) / (2.0f * logf(base));
}

/* rope.rs:128-172, x = [n_head][head_dim], the last n_rot lanes of each head
 * rotated in pairs. */
void rkvo_rope_yarn_tail(float* x, uint32_t n_head, uint32_t head_dim, uint32_t n_rot, uint32_t pos,
                         uint64_t n_ctx_orig, float freq_base, float freq_scale, float ext_factor, float attn_factor,
                         float beta_fast, float beta_slow, int inverse) {
    uint32_t n_nope = head_dim - n_rot;
    float theta_scale = powf(freq_base, -2.0f / (float)n_rot);
    float sin_sign = inverse ? -1.0f : 1.0f;
    float corr0 = 0.0f, corr1 = 0.0f;
    if (ext_factor != 0.0f) {
        corr0 = fmaxf(floorf(yarn_corr_dim((int32_t)n_rot, n_ctx_orig, beta_fast, freq_base)), 0.0f);
        corr1 = fminf(ceilf(yarn_corr_dim((int32_t)n_rot, n_ctx_orig, beta_slow, freq_base)), (float)((int32_t)n_rot - 1));
    }
    for (uint32_t h = 0; h < n_head; ++h) {
        float* tail = x + (size_t)h * head_dim + n_nope;
        float theta_extrap = (float)pos;
        for (uint32_t i = 0; i < n_rot; i += 2) {
            float theta_interp = freq_scale * theta_extrap;
            float theta = theta_interp;
            float mscale = attn_factor;
            if (ext_factor != 0.0f) {
                float ramp_mix = yarn_ramp(corr0, corr1, (int32_t)i) * ext_factor;
                theta = theta_interp * (1.0f - ramp_mix) + theta_extrap * ramp_mix;
                mscale *= 1.0f + 0.1f * logf(1.0f / freq_scale);
            }
            float c = cosf(theta) * mscale;
            float s = sin_sign * sinf(theta) * mscale;
            float x0 = tail[i], x1 = tail[i + 1];
            tail[i] = x0 * c - x1 * s;
            tail[i + 1] = x0 * s + x1 * c;
            theta_extrap *= theta_scale;
        }
    }
}

/* compressor.rs:284-330: RMSNorm with an f64 sum of squares (DSV4_RMS_EPS
 * 1e-6), then the YaRN rotation of the last 64 lanes with
 * compress_rope_params (compressor.rs:372-397) at comp_pos. */
/* The compressed-layer rotation alone (compress_rope_params,
 * compressor.rs:372-397) of the last 64 lanes of a head_dim row. */
void rkvo_compress_rope(float* row, int64_t head_dim, uint32_t comp_pos) {
    const float scale_factor = 16.0f, freq_scale = 1.0f / scale_factor;
    const float attn_factor = 1.0f / (1.0f + 0.1f * logf(1.0f / freq_scale));
    rkvo_rope_yarn_tail(row, 1, (uint32_t)head_dim, ROPE, comp_pos, 65536, 160000.0f, freq_scale, 1.0f, attn_factor,
                        32.0f, 1.0f, 0);
}

void rkvo_compressor_postprocess(float* row, int64_t head_dim, const float* norm, uint32_t comp_pos) {
    double ss = 0.0;
    for (int64_t j = 0; j < head_dim; ++j) ss += (double)row[j] * (double)row[j];
    float rms = 1.0f / sqrtf((float)(ss / (double)head_dim) + 1e-6f);
    for (int64_t j = 0; j < head_dim; ++j) row[j] = row[j] * rms * norm[j];
    rkvo_compress_rope(row, head_dim, comp_pos);
}

typedef struct {
    uint8_t* pool; int64_t n_pages; int32_t n_layers; int32_t layer; int32_t ratio;
    float* state_kv; float* state_score; uint32_t* state_count; int64_t n_states;
    const float* kv; const float* score; int64_t n_tok; const int32_t* pos; const int32_t* state_of;
    const int32_t* emit_slot; const float* ape; const float* norm;
    int32_t t_id, n_workers; uint32_t status;
} cmp_job;

static void* cmp_worker(void* p) {
    cmp_job* j = (cmp_job*)p;
    int64_t coff = cmp_coff(j->ratio), width = coff * ROW_DIM, state_floats = coff * j->ratio * width;
    float* sc = (float*)malloc((size_t)width * 4);
    float row[ROW_DIM];
    uint8_t codes[LATENT];
    float scales[NBLK];
    uint16_t rope[ROPE];
    for (int64_t t = 0; t < j->n_tok; ++t) {
        int32_t s = j->state_of[t], pos = j->pos[t];
        if (s < 0 || s >= j->n_states || pos < 0) { if (j->t_id == 0) j->status |= 1u << RKVO_INDEX_OUT_OF_RANGE; continue; }
        if (s % j->n_workers != j->t_id) continue;
        /* compressor.rs:264-269: sc_cur += ape column pos % ratio */
        memcpy(sc, j->score + t * width, (size_t)width * 4);
        if (j->ape)
            for (int64_t c = 0; c < width; ++c) sc[c] += j->ape[(int64_t)(pos % j->ratio) * width + c];
        if (!rkvo_compressor_accumulate(j->state_kv + s * state_floats, j->state_score + s * state_floats,
                                        j->state_count + s, j->ratio, ROW_DIM, j->kv + t * width, sc, row))
            continue;
        int32_t slot = j->emit_slot[t];
        if (slot < 0) continue;
        int64_t page = slot / PAGE_TOKENS, off = slot % PAGE_TOKENS;
        if (page >= j->n_pages) { j->status |= 1u << RKVO_INDEX_OUT_OF_RANGE; continue; }
        uint32_t comp_pos = (uint32_t)pos + 1 >= (uint32_t)j->ratio ? (uint32_t)pos + 1 - (uint32_t)j->ratio : 0;
        rkvo_compressor_postprocess(row, ROW_DIM, j->norm, comp_pos);
        int rc = rkvo_quantize_row_f32(row, ROW_DIM, ROPE, codes, scales, rope);
        if (rc != RKVO_OK) { j->status |= 1u << rc; continue; }
        uint8_t* pg = page_ptr(j->pool, j->n_pages, j->layer, page);
        memcpy(pg + off * LATENT, codes, LATENT);
        memcpy(pg + CODES_BYTES + off * NBLK * 4, scales, NBLK * 4);
        memcpy(pg + CODES_BYTES + SCALES_BYTES + off * ROPE * 2, rope, ROPE * 2);
    }
    free(sc);
    return NULL;
}

/* One compressor step for a batch of tokens (576-lane rows; kv, score
 * [n_tok][coff*576]; ape [ratio][coff*576] or NULL; norm [576]), token by
 * token in input order over the reference-layout states
 * (state_kv/state_score [n_states][coff*ratio][coff*576], state_count
 * [n_states]).  A row emitted by token t is post-processed, quantized and
 * stored at emit_slot[t] (< 0: dropped).  States are split over threads. */
uint32_t rkvo_compress_append(uint8_t* pool, int64_t n_pages, int32_t n_layers, int32_t layer, int32_t ratio,
                              float* state_kv, float* state_score, uint32_t* state_count, int64_t n_states,
                              const float* kv, const float* score, int64_t n_tok, const int32_t* pos,
                              const int32_t* state_of, const int32_t* emit_slot, const float* ape, const float* norm,
                              int n_threads) {
    if (n_tok <= 0) return 0;
    if (layer < 0 || layer >= n_layers) return 1u << RKVO_INVALID_LAYER;
    if (ratio <= 0) return 1u << RKVO_SHAPE_MISMATCH;
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    if (n_states > 0 && n_threads > n_states) n_threads = (int)n_states;
    pthread_t th[256];
    cmp_job jobs[256];
    for (int t = 0; t < n_threads; ++t) {
        jobs[t] = (cmp_job){pool, n_pages, n_layers, layer, ratio, state_kv, state_score, state_count, n_states,
                            kv, score, n_tok, pos, state_of, emit_slot, ape, norm, t, n_threads, 0};
        if (n_threads == 1) cmp_worker(&jobs[t]);
        else pthread_create(&th[t], NULL, cmp_worker, &jobs[t]);
    }
    uint32_t st = 0;
    for (int t = 0; t < n_threads; ++t) {
        if (n_threads > 1) pthread_join(th[t], NULL);
        st |= jobs[t].status;
    }
    return st;
}

/* The indexer pool's compressor step (attention.rs:405-429 calls
 * compressor_decode_one on the indexer pool, head_dim 128): the same APE
 * bias, accumulate_wide / maybe_emit window (compressed.rs:310-417), per-
 * dimension softmax aggregate (:481-554), RMSNorm with an f64 sum of squares
 * and RoPE of the last 64 lanes at pos + 1 - ratio (compressor.rs:284-330),
 * for 128-lane rows (kv, score [n_tok][coff*128]; ape [ratio][coff*128] or
 * NULL; norm [128]).  The row emitted by token t is written as f32 to
 * out_rows[emit_row[t]] (< 0: dropped; >= n_out_rows: INDEX_OUT_OF_RANGE),
 * before the indexer's Hadamard + FP4 QAT step (compressor.rs:343-348), which
 * is not restated here.  States [n_states][coff*ratio][coff*128]. */
#define IDX_DIM 128
typedef struct {
    float* out_rows; int64_t n_out_rows; int32_t ratio;
    float* state_kv; float* state_score; uint32_t* state_count; int64_t n_states;
    const float* kv; const float* score; int64_t n_tok; const int32_t* pos; const int32_t* state_of;
    const int32_t* emit_row; const float* ape; const float* norm;
    int32_t t_id, n_workers; uint32_t status;
} icmp_job;

static void* icmp_worker(void* p) {
    icmp_job* j = (icmp_job*)p;
    int64_t coff = cmp_coff(j->ratio), width = coff * IDX_DIM, state_floats = coff * j->ratio * width;
    float sc[2 * IDX_DIM];
    float row[IDX_DIM];
    for (int64_t t = 0; t < j->n_tok; ++t) {
        int32_t s = j->state_of[t], pos = j->pos[t];
        if (s < 0 || s >= j->n_states || pos < 0) { if (j->t_id == 0) j->status |= 1u << RKVO_INDEX_OUT_OF_RANGE; continue; }
        if (s % j->n_workers != j->t_id) continue;
        memcpy(sc, j->score + t * width, (size_t)width * 4);
        if (j->ape)
            for (int64_t c = 0; c < width; ++c) sc[c] += j->ape[(int64_t)(pos % j->ratio) * width + c];
        if (!rkvo_compressor_accumulate(j->state_kv + s * state_floats, j->state_score + s * state_floats,
                                        j->state_count + s, j->ratio, IDX_DIM, j->kv + t * width, sc, row))
            continue;
        int32_t r = j->emit_row[t];
        if (r < 0) continue;
        if (r >= j->n_out_rows) { j->status |= 1u << RKVO_INDEX_OUT_OF_RANGE; continue; }
        uint32_t comp_pos = (uint32_t)pos + 1 >= (uint32_t)j->ratio ? (uint32_t)pos + 1 - (uint32_t)j->ratio : 0;
        rkvo_compressor_postprocess(row, IDX_DIM, j->norm, comp_pos);
        memcpy(j->out_rows + (int64_t)r * IDX_DIM, row, sizeof(row));
    }
    return NULL;
}

uint32_t rkvo_indexer_compress_append(float* out_rows, int64_t n_out_rows, int32_t ratio, float* state_kv,
                                      float* state_score, uint32_t* state_count, int64_t n_states, const float* kv,
                                      const float* score, int64_t n_tok, const int32_t* pos, const int32_t* state_of,
                                      const int32_t* emit_row, const float* ape, const float* norm, int n_threads) {
    if (n_tok <= 0) return 0;
    if (ratio <= 0 || cmp_coff(ratio) * ratio > 128) return 1u << RKVO_SHAPE_MISMATCH;
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    if (n_states > 0 && n_threads > n_states) n_threads = (int)n_states;
    pthread_t th[256];
    icmp_job jobs[256];
    for (int t = 0; t < n_threads; ++t) {
        jobs[t] = (icmp_job){out_rows, n_out_rows, ratio, state_kv, state_score, state_count, n_states, kv, score,
                             n_tok, pos, state_of, emit_row, ape, norm, t, n_threads, 0};
        if (n_threads == 1) icmp_worker(&jobs[t]);
        else pthread_create(&th[t], NULL, icmp_worker, &jobs[t]);
    }
    uint32_t st = 0;
    for (int t = 0; t < n_threads; ++t) {
        if (n_threads > 1) pthread_join(th[t], NULL);
        st |= jobs[t].status;
    }
    return st;
}

/* The host libm's expf over an array (the reference's f32::exp), for checking
 * the product's expf rounding exhaustively. */
typedef struct { const float* x; float* out; int64_t b, e; } expf_job;
static void* expf_worker(void* p) {
    expf_job* j = (expf_job*)p;
    for (int64_t i = j->b; i < j->e; ++i) j->out[i] = expf(j->x[i]);
    return NULL;
}
void rkvo_expf_batch(const float* x, float* out, int64_t n, int n_threads) {
    if (n <= 0) return;
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    pthread_t th[256];
    expf_job jobs[256];
    for (int t = 0; t < n_threads; ++t) {
        jobs[t] = (expf_job){x, out, n * t / n_threads, n * (t + 1) / n_threads};
        if (n_threads == 1) expf_worker(&jobs[t]);
        else pthread_create(&th[t], NULL, expf_worker, &jobs[t]);
    }
    if (n_threads > 1)
        for (int t = 0; t < n_threads; ++t) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------------ */
/* indexer.rs:198-216, the scoring of compressed indexer rows                */
/* ------------------------------------------------------------------------ */

#define IDX_HEADS 64
#define IDX_DIM 128

/* score of one 128-lane row against q [64][128] and w [64]: per head a dot
 * accumulated lane by lane, ReLU, then the weighted sum head by head, f32
 * throughout (no contraction). */
float rkvo_indexer_score_row(const float* row, const float* q, const float* w) {
    float s = 0.0f;
    for (int h = 0; h < IDX_HEADS; ++h) {
        const float* qh = q + h * IDX_DIM;
        float dot = 0.0f;
        for (int i = 0; i < IDX_DIM; ++i) dot += row[i] * qh[i];
        if (dot > 0.0f) s += dot * w[h];
    }
    return s;
}

typedef struct {
    const float* rows; const int64_t* row_start; const int32_t* seq_rows; int64_t n_seq;
    const float* q; const float* w; const int32_t* seq_of_query; const int32_t* n_visible;
    float* scores; int64_t ld; int32_t q0, q1; uint32_t status;
} idx_job;

static void* idx_worker(void* p) {
    idx_job* j = (idx_job*)p;
    for (int32_t qi = j->q0; qi < j->q1; ++qi) {
        int32_t s = j->seq_of_query[qi], nv = j->n_visible[qi];
        if (s < 0 || s >= j->n_seq || nv < 0 || nv > j->seq_rows[s]) { j->status |= 1u << RKVO_INDEX_OUT_OF_RANGE; continue; }
        const float* base = j->rows + j->row_start[s] * IDX_DIM;
        for (int32_t c = 0; c < nv; ++c)
            j->scores[(int64_t)qi * j->ld + c] =
                rkvo_indexer_score_row(base + (int64_t)c * IDX_DIM, j->q + (int64_t)qi * IDX_HEADS * IDX_DIM,
                                       j->w + (int64_t)qi * IDX_HEADS);
    }
    return NULL;
}

/* Scores of a batch of queries (rkv_indexer_scores_f32's contract), threads
 * over queries; returns the status bits. */
uint32_t rkvo_indexer_scores(const float* rows, const int64_t* row_start, const int32_t* seq_rows, int64_t n_seq,
                             const float* q, const float* w, const int32_t* seq_of_query, const int32_t* n_visible,
                             int32_t n_q, float* scores, int64_t ld, int n_threads) {
    if (n_q <= 0) return 0;
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    if (n_threads > n_q) n_threads = n_q;
    pthread_t th[256];
    idx_job jobs[256];
    for (int t = 0; t < n_threads; ++t) {
        jobs[t] = (idx_job){rows, row_start, seq_rows, n_seq, q, w, seq_of_query, n_visible, scores, ld,
                            (int32_t)((int64_t)n_q * t / n_threads), (int32_t)((int64_t)n_q * (t + 1) / n_threads), 0};
        if (n_threads == 1) idx_worker(&jobs[t]);
        else pthread_create(&th[t], NULL, idx_worker, &jobs[t]);
    }
    uint32_t st = 0;
    for (int t = 0; t < n_threads; ++t) {
        if (n_threads > 1) pthread_join(th[t], NULL);
        st |= jobs[t].status;
    }
    return st;
}
