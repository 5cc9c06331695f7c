"""The oracle's restatement of the reference's quantised formats, pinned to
the reference's own tests (src/kernels.rs:349-437): f16 conversion known
answers, Q8_0 dequantisation exact, Q6_K and Q4_K dequantisation consistent
with their quantised dot products, block sizes. CPU only."""
import numpy as np

from oracle import oracle as orc


def test_f16_to_f32_known_answers():
    # kernels.rs:352-376
    cases = [(0x0000, 0.0), (0x0001, 5.9604645e-8), (0x0200, 3.0517578e-5),
             (0x03FF, 6.097555e-5), (0x0400, 6.1035156e-5), (0x3C00, 1.0), (0xC000, -2.0),
             (0x8001, -5.9604645e-8)]
    for h, want in cases:
        got = orc.f16_to_f32(h)
        assert abs(got - want) <= abs(want) * 1e-6, (hex(h), got, want)
    assert np.isinf(orc.f16_to_f32(0x7C00)) and np.isnan(orc.f16_to_f32(0x7C01))
    for h in range(0, 1 << 16, 7):  # every 7th half against numpy's conversion
        want = np.array([h], np.uint16).view(np.float16).astype(np.float32)[0]
        got = np.float32(orc.f16_to_f32(h))
        assert (np.isnan(got) and np.isnan(want)) or got == want, hex(h)


def test_block_sizes():
    # kernels.rs:380-384
    assert orc.row_bytes(orc.QTYPE_Q4_K, 256) == 144
    assert orc.row_bytes(orc.QTYPE_Q6_K, 256) == 210


def test_dequantize_q8_0_row_exact():
    # kernels.rs:386-398: two blocks, d = 0.5 (0x3800), quants blk*32 + i - 40.
    b = bytearray()
    for blk in range(2):
        b += (0x3800).to_bytes(2, "little")
        b += bytes(((blk * 32 + i - 40) & 0xFF) for i in range(32))
    out = orc.dequantize(orc.QTYPE_Q8_0, np.frombuffer(bytes(b), np.uint8), 1, 64)[0]
    assert (out == 0.5 * (np.arange(64) - 40)).all()


def _q8_test_vector():
    qs = np.clip(np.arange(256) * 3 - 128, -128, 127).astype(np.int8)
    bs = qs.reshape(16, 16).astype(np.int16).sum(axis=1).astype(np.int16)
    return np.array([1 / 127], np.float32), qs, bs


def test_q6k_dequantize_matches_dot():
    # kernels.rs:401-424
    blk = bytearray(210)
    for i in range(128):
        blk[i] = (i * 7 + 3) & 0xFF
    for i in range(64):
        blk[128 + i] = (i * 13 + 5) & 0xFF
    for i in range(16):
        blk[192 + i] = i + 1
    blk[208:210] = (0x3C00).to_bytes(2, "little")
    d, qs, _ = _q8_test_vector()
    dot = orc.vec_dot_q6k_q8k(np.frombuffer(bytes(blk), np.uint8), d, qs)
    deq = orc.dequantize(orc.QTYPE_Q6_K, np.frombuffer(bytes(blk), np.uint8), 1, 256)[0]
    dot_ref = float((deq * qs.astype(np.float32) / 127.0).sum())
    assert abs(dot - dot_ref) / max(abs(dot), 1e-6) < 1e-4


def test_q4k_dequantize_matches_dot():
    # kernels.rs:427-437 (non-zero dot), plus the same consistency check as Q6_K.
    blk = bytearray(144)
    blk[0:2] = (0x3C00).to_bytes(2, "little")
    blk[2:4] = (0x3800).to_bytes(2, "little")
    for i in range(12):
        blk[4 + i] = (i * 5 + 1) & 0x3F
    for i in range(128):
        blk[16 + i] = (i * 7 + 3) & 0xFF
    d, qs, bs = _q8_test_vector()
    w = np.frombuffer(bytes(blk), np.uint8)
    dot = orc.vec_dot_q4k_q8k(w, d, qs, bs)
    assert np.isfinite(dot) and abs(dot) > 1e-6
    deq = orc.dequantize(orc.QTYPE_Q4_K, w, 1, 256)[0]
    dot_ref = float((deq.astype(np.float64) * qs / 127.0).sum())
    assert abs(dot - dot_ref) / max(abs(dot), 1e-6) < 1e-4


def test_q8k_quantization_round_trip():
    rng = np.random.default_rng(3)
    x = rng.standard_normal(512).astype(np.float32)
    d, qs, bs = orc.quantize_row_q8k(x)
    back = (qs.reshape(2, 256) * d[:, None]).reshape(-1)
    assert np.abs(back - x).max() <= np.abs(x).max() / 127.0
    assert (bs == qs.reshape(-1, 16).astype(np.int32).sum(axis=1)).all()
