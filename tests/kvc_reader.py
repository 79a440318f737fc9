"""Independent reader and header writer of the KVC file format (test
infrastructure), restated from rsLLM's plan (docs/03-HLD.md:242-282) as this
repository pins it: 48-byte little-endian header, length-prefixed rendered
text, the "DSV4" engine payload with the token ids and every page of every
layer as stored in the pool."""
import struct

import numpy as np

PAGE_BYTES = 43008
HEADER = struct.Struct("<3sBIIQQQQI")  # magic, version, quant_bits, reason, token_count, ctx_size, created_at,
                                      # payload_bytes, reserved
PAYLOAD = struct.Struct("<7I")        # magic, version, vocab_size, n_layers, head_dim, page_tokens, n_pages
assert HEADER.size == 48


def read(path: str) -> dict:
    data = open(path, "rb").read()
    (magic, version, quant_bits, reason, token_count, ctx_size, created_at, payload_bytes,
     reserved) = HEADER.unpack_from(data, 0)
    off = HEADER.size
    (text_len,) = struct.unpack_from("<I", data, off)
    off += 4
    text = data[off:off + text_len]
    off += text_len
    pm, pv, vocab, n_layers, head_dim, page_tokens, n_pages = PAYLOAD.unpack_from(data, off)
    off += PAYLOAD.size
    tokens = np.frombuffer(data, "<u4", token_count, off).astype(np.int64).astype(np.int32)
    off += 4 * token_count
    pages = np.frombuffer(data, np.uint8, n_layers * n_pages * PAGE_BYTES, off).reshape(n_layers, n_pages, PAGE_BYTES)
    off += pages.size
    return dict(magic=magic, version=version, quant_bits=quant_bits, reason=reason, token_count=token_count,
                ctx_size=ctx_size, created_at=created_at, payload_bytes=payload_bytes, reserved=reserved, text=text,
                payload_magic=pm, payload_version=pv, vocab_size=vocab, n_layers=n_layers, head_dim=head_dim,
                page_tokens=page_tokens, n_pages=n_pages, tokens=tokens, pages=pages,
                body_bytes=len(data) - HEADER.size, trailing=len(data) - off)


def write_header(path: str, magic=b"KVC", version=1, quant_bits=8, reason=0, token_count=1, ctx_size=64,
                 created_at=0, payload_bytes=0, extra: bytes = b"") -> None:
    with open(path, "wb") as f:
        f.write(HEADER.pack(magic, version, quant_bits, reason, token_count, ctx_size, created_at, payload_bytes, 0))
        f.write(extra)
