"""Pins the CPU oracle to the reference: every integer result must match the
reference's own quantizers (import_params.py:229-248, run by
tests/golden/make_golden.py) and its shipped int8 export bit for bit."""
import hashlib
import os

import numpy as np
import pytest

G = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def qg():
    return np.load(os.path.join(G, "quant_golden.npz"))


@pytest.mark.parametrize("name", ["a", "b", "c"])
def test_quantize_int8_matches_reference(oracle, qg, name):
    q, s = oracle.quantize_int8(qg[f"{name}_w"])
    np.testing.assert_array_equal(q, qg[f"{name}_q8"])
    np.testing.assert_array_equal(s, qg[f"{name}_s8"])


@pytest.mark.parametrize("name", ["a", "b", "c"])
@pytest.mark.parametrize("group", [32, 128])
def test_quantize_int4_matches_reference(oracle, qg, name, group):
    p, d = oracle.quantize_int4(qg[f"{name}_w"], group)
    np.testing.assert_array_equal(p, qg[f"{name}_p4_g{group}"])
    np.testing.assert_array_equal(d, qg[f"{name}_d4_g{group}"])


def test_config1_quantization_digest(oracle, qg):
    """W ~ N(0, 0.02) [1024, 1024], x ~ N(0, 1), seed 0."""
    rng = np.random.default_rng(0)
    x1 = rng.standard_normal((1, 1024)).astype(np.float32)
    w1 = (rng.standard_normal((1024, 1024)) * 0.02).astype(np.float32)
    np.testing.assert_array_equal(x1, qg["c1_x"])
    q, s = oracle.quantize_int8(w1)
    np.testing.assert_array_equal(q[:16], qg["c1_q8_head"])
    np.testing.assert_array_equal(s, qg["c1_s8"])
    assert hashlib.sha256(q.tobytes()).digest() == qg["c1_q8_sha256"].tobytes()


def test_dequant_int8_real_export(oracle):
    """Real `--quant int8` export shipped with the reference: unpack + dequant bit-exact."""
    ex = np.load(os.path.join(G, "int8_export.npz"))
    q, s = ex["q"], ex["s"]
    rows, cols = q.shape
    deq = oracle.dequant(q, s, "int8", rows, cols)
    np.testing.assert_array_equal(deq.view(np.uint32), ex["deq"].view(np.uint32))
    # every row of the real export saturates at |q| = 127 (per-row absmax)
    assert (ex["row_absmax"] == 127).all()


def test_dequant_int4_matches_numpy_formula(oracle, qg):
    w = qg["b_w"]
    for group in (32, 128):
        p, d = qg[f"b_p4_g{group}"], qg[f"b_d4_g{group}"]
        deq = oracle.dequant(p, d, "int4", w.shape[0], w.shape[1], group)
        lo = (p & 0xF).astype(np.float32) - 8.0
        hi = (p >> 4).astype(np.float32) - 8.0
        nib = np.empty(w.shape, np.float32)
        nib[:, 0::2], nib[:, 1::2] = lo, hi
        ref = nib * np.repeat(d.view(np.float16).astype(np.float32), group, axis=1)
        np.testing.assert_array_equal(deq.view(np.uint32), ref.view(np.uint32))


def test_f32_to_f16_matches_numpy(oracle):
    f = np.load(os.path.join(G, "f16_golden.npz"))
    got = np.array([oracle.f32_to_f16_bits(v) for v in f["x"]], np.uint16)
    np.testing.assert_array_equal(got, f["h"])


def _argmax_tree(lg):
    """Independent pure-Python restatement of ArgMax (Gemma3CS.compute:911-928)."""
    val, idx = [], []
    for t in range(256):
        bv, bi = -3.0e38, 0
        for i in range(t, len(lg), 256):
            if lg[i] > bv:
                bv, bi = float(lg[i]), i
        val.append(bv)
        idx.append(bi)
    s = 128
    while s > 0:
        for t in range(s):
            if val[t + s] > val[t]:
                val[t], idx[t] = val[t + s], idx[t + s]
        s //= 2
    return idx[0]


def test_argmax_tie_break(oracle):
    """Ties resolve by the reference's thread tree, not by lowest index."""
    lg = np.zeros(1000, np.float32)
    lg[700] = 5.0
    lg[3] = 5.0
    assert oracle.argmax(lg) == _argmax_tree(lg) == 700
    lg = np.zeros(1000, np.float32)
    lg[260] = 5.0          # same thread (4) as index 4: first strict max in its stride wins
    lg[4] = 5.0
    assert oracle.argmax(lg) == _argmax_tree(lg) == 4
    rng = np.random.default_rng(3)
    for _ in range(20):
        lg = rng.integers(0, 4, 3000).astype(np.float32)   # many ties
        assert oracle.argmax(lg) == _argmax_tree(lg)


def test_gemv_matches_float64(oracle, qg):
    w = qg["c_w"]
    rng = np.random.default_rng(1)
    x = rng.standard_normal((3, w.shape[1])).astype(np.float32)
    for quant, group in (("int8", 0), ("int4", 32), ("int4", 128)):
        if quant == "int8":
            wq, s = qg["c_q8"], qg["c_s8"]
        else:
            wq, s = qg[f"c_p4_g{group}"], qg[f"c_d4_g{group}"]
        deq = oracle.dequant(wq, s, quant, w.shape[0], w.shape[1], group or 32)
        y = oracle.gemv(x, wq, s, quant, w.shape[0], group or 32)
        ref = x.astype(np.float64) @ deq.astype(np.float64).T
        np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-5)


def _kv_int8_numpy(x):
    """Independent numpy restatement of WriteCacheFull's INT8 variant (G3CS:300-380) in
    IEEE fp32: the oracle's C version must agree with it bit for bit."""
    x = x.astype(np.float32)
    mn, mx = x.min(axis=-1), x.max(axis=-1)
    scale = ((mx - mn) / np.float32(255.0)).astype(np.float32)
    scale = np.where(scale < np.float32(1e-9), np.float32(1e-9), scale).astype(np.float32)
    zp = np.clip(np.rint((-mn / scale).astype(np.float32)), 0, 255).astype(np.float32)
    inv = (np.float32(1.0) / scale).astype(np.float32)
    q = np.clip(np.rint((x * inv[..., None]).astype(np.float32)) + zp[..., None], 0, 255).astype(np.uint8)
    sz = (scale.astype(np.float16).view(np.uint16).astype(np.uint32)
          | (zp.astype(np.float16).view(np.uint16).astype(np.uint32) << 16))
    return q, sz


def test_kv_write_int8_oracle_matches_numpy_restatement(oracle):
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((40, 4, 64)) * 3).astype(np.float32)
    x[0, 0] = 0.5                                        # constant row: scale floor, fp16 scale 0
    x[1, 1] = np.abs(x[1, 1]) + 2                        # all positive: zp 0
    x[2, 2] = -np.abs(x[2, 2]) - 2                       # all negative: zp clamps to 255
    x[3, 3] = (np.arange(64) - 32).astype(np.float32) / 255.0
    q, sz = oracle.kv_write_int8(x, 4, 64)
    qn, szn = _kv_int8_numpy(x)
    np.testing.assert_array_equal(q, qn)
    np.testing.assert_array_equal(sz, szn)
    # kv_unpack8 round trip: within half a step for rows whose range holds 0
    d = oracle.kv8_dequant(q, sz)
    ok = (x.min(-1) <= 0) & (x.max(-1) >= 0) & (np.ptp(x, axis=-1) > 1e-3)
    step = (sz & 0xFFFF).astype(np.uint16).view(np.float16).astype(np.float32)
    assert np.all(np.abs(d - x)[ok] <= (step[ok][:, None] * 0.5 + np.abs(x[ok]) * 2e-3 + 1e-6))
