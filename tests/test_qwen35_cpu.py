"""The oracle's restatement of ApplyRopePartial (Qwen3_5CS.compute:367-393) against an
element-by-element reading of the reference kernel in fp32, and its agreement with the
full split-half rotation when every dim rotates (no GPU)."""
import numpy as np

from oracle import oracle as orc


def _rope_partial_loop(x, rot, pos0, cos_t, sin_t):
    out = x.astype(np.float32).copy()
    seq, heads, hd = out.shape
    r2 = rot // 2
    c = cos_t.reshape(-1).view(np.float16).astype(np.float32)
    s = sin_t.reshape(-1).view(np.float16).astype(np.float32)
    for l in range(seq):
        for h in range(heads):
            for i in range(r2):
                x1, x2 = out[l, h, i], out[l, h, i + r2]
                cc, ss = c[(pos0 + l) * r2 + i], s[(pos0 + l) * r2 + i]
                out[l, h, i] = np.float32(x1 * cc - x2 * ss)
                out[l, h, i + r2] = np.float32(x2 * cc + x1 * ss)
    return out


def test_partial_rope_matches_the_kernel_reading():
    rng = np.random.default_rng(5)
    seq, heads, hd, rot, pos0 = 3, 2, 128, 32, 7
    x = rng.standard_normal((seq, heads, hd)).astype(np.float32)
    cos_t, sin_t = orc.rope_table(64, rot, 10_000_000.0)      # inv_freq over the rotated dims
    got = orc.rope_apply_partial(x.copy(), heads, hd, rot, pos0, cos_t, sin_t).reshape(seq, heads, hd)
    ref = _rope_partial_loop(x, rot, pos0, cos_t, sin_t)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    assert np.array_equal(got[:, :, rot:], x[:, :, rot:])       # dims >= rot untouched


def test_partial_rope_over_all_dims_is_the_full_rotation():
    rng = np.random.default_rng(6)
    seq, heads, hd, pos0 = 2, 3, 64, 5
    x = rng.standard_normal((seq, heads, hd)).astype(np.float32)
    cos_t, sin_t = orc.rope_table(32, hd, 10000.0)
    a = orc.rope_apply_partial(x.copy(), heads, hd, hd, pos0, cos_t, sin_t).reshape(-1)
    b = orc.rope_apply(x.copy(), heads, hd, pos0, cos_t, sin_t).reshape(-1)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
