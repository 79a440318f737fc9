"""KVC file naming and header handling on the host (no GPU): the file name is
SHA1 of the token ids as little-endian u32 (docs/03-HLD.md: "SHA1(token_ids)"),
checked against hashlib across SHA-1's padding boundaries; headers written by
the independent test writer are read back field by field, and malformed
files are rejected with rsLLM's error kinds."""
import hashlib

import numpy as np
import pytest

import rsllm_b200 as rk
from rsllm_b200.prefix_pool import kvc_name, read_kvc_header

import kvc_reader


@pytest.mark.parametrize("n", [0, 1, 13, 14, 15, 16, 17, 31, 32, 33, 1000, 8229])
def test_name_is_sha1_of_little_endian_ids(n):
    rng = np.random.default_rng(n)
    t = rng.integers(-2**31, 2**31, n, dtype=np.int64).astype(np.int32)
    assert kvc_name(t) == hashlib.sha1(t.astype("<u4").tobytes()).hexdigest() + ".kvc"


def test_header_fields_round_trip(tmp_path):
    p = str(tmp_path / "a.kvc")
    kvc_reader.write_header(p, reason=2, token_count=8229, ctx_size=8256, created_at=1_700_000_000,
                            payload_bytes=12345)
    h = read_kvc_header(p)
    assert h == dict(version=1, quant_bits=8, reason=2, reserved=0, token_count=8229, ctx_size=8256,
                     created_at=1_700_000_000, payload_bytes=12345)


@pytest.mark.parametrize("case", ["magic", "version", "quant_bits", "short"])
def test_malformed_headers_are_rejected(tmp_path, case):
    p = str(tmp_path / "b.kvc")
    if case == "short":
        open(p, "wb").write(b"KVC\x01")
    else:
        kw = {"magic": dict(magic=b"KVX"), "version": dict(version=2), "quant_bits": dict(quant_bits=4)}[case]
        kvc_reader.write_header(p, **kw)
    with pytest.raises(rk.InvalidArgument):
        read_kvc_header(p)
    with pytest.raises(rk.InvalidArgument):
        read_kvc_header(str(tmp_path / "missing.kvc"))
