"""The KV-cache wire format's host-side check (q3a_kv_wire_check), no GPU:
blobs built here with an independent numpy restatement of the format and
its checksum are accepted; a flipped payload bit, a wrong field, a short
blob and a foreign magic are refused."""
import struct

import numpy as np
import pytest

import q3attn

HEADER = "<IHHHHHHHHIIIQQ16x"   # the 64-byte q3a_kv_wire_header
GOLDEN = np.uint64(0x9E3779B97F4A7C15)


def mix(z):
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def checksum(payload: bytes) -> int:
    w = np.frombuffer(payload, dtype="<u8")
    with np.errstate(over="ignore"):
        i = np.arange(w.size, dtype=np.uint64)
        return int(mix(w + i * GOLDEN).sum(dtype=np.uint64))


def blob(dtype=1, n_layers=2, heads=(2, 3), n_kv=8, pos0=5, n_tok=7, seed=0):
    es = 2 if dtype == 1 else 4
    pay = n_layers * heads[1] * 2 * n_tok * 128 * es
    payload = np.random.default_rng(seed).integers(0, 256, pay, dtype=np.uint8).tobytes()
    hdr = struct.pack(HEADER, q3attn.KV_WIRE_MAGIC, q3attn.KV_WIRE_VERSION, dtype, 128, n_kv,
                      heads[0], heads[1], 3, n_layers, pos0, n_tok, 0, pay, checksum(payload))
    assert len(hdr) == q3attn.KV_WIRE_HEADER_BYTES
    return bytearray(hdr + payload)


@pytest.mark.parametrize("dtype", [0, 1])
def test_well_formed_blobs_pass(dtype):
    q3attn.kv_wire_check(blob(dtype=dtype))
    q3attn.kv_wire_check(blob(dtype=dtype, n_layers=1, heads=(0, 8), n_tok=1, seed=3))


def test_flipped_payload_bit_is_refused():
    b = blob()
    for off in (64, 64 + 1000, len(b) - 1):
        c = bytearray(b)
        c[off] ^= 0x10
        with pytest.raises(q3attn.Q3AError, match="checksum"):
            q3attn.kv_wire_check(c)


def test_swapped_words_are_refused():
    """The checksum is a sum, but every word is mixed with its index, so
    exchanging two payload words changes it."""
    b = blob()
    c = bytearray(b)
    c[64:72], c[72:80] = b[72:80], b[64:72]
    assert c != b
    with pytest.raises(q3attn.Q3AError, match="checksum"):
        q3attn.kv_wire_check(c)


@pytest.mark.parametrize("field,value", [(0, 0x12345678), (1, 2), (2, 7), (3, 64),
                                          (6, 0), (5, 7), (12, 10)])
def test_bad_header_fields_are_refused(field, value):
    b = blob()
    f = list(struct.unpack(HEADER, bytes(b[:64])))
    f[field] = value
    b[:64] = struct.pack(HEADER, *f)
    with pytest.raises(q3attn.Q3AError):
        q3attn.kv_wire_check(b)


def test_short_blob_is_refused():
    b = blob()
    with pytest.raises(q3attn.Q3AError):
        q3attn.kv_wire_check(b[:-16])
    with pytest.raises(q3attn.Q3AError):
        q3attn.kv_wire_check(b[:32])
