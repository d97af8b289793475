"""The oracle's restatement of the repetition / presence penalty
(ApplyRepetitionPresencePenalty, Qwen3_5CS.compute:1421-1433) and of
MarkSampledTokenSeen (:1436-1441), against an element-by-element reading of
the reference kernel in fp32 (no GPU)."""
import numpy as np

from oracle import oracle as orc


def _reference_loop(logits, seen, presence, repetition):
    out = logits.astype(np.float32).copy()
    rep, pres = np.float32(repetition), np.float32(presence)
    for i in range(out.shape[-1]):
        if seen[i] == 0:
            continue
        l = out[i]
        l = l / rep if l > np.float32(0) else l * rep
        out[i] = np.float32(l - pres)
    return out


def test_penalty_restatement_matches_the_kernel_reading():
    rng = np.random.default_rng(3)
    V = 257
    logits = (rng.standard_normal(V) * 4).astype(np.float32)
    logits[:5] = [0.0, -0.0, 1e-30, -1e-30, 3.0]
    seen = (rng.random(V) < 0.3).astype(np.uint32) * rng.integers(1, 4, V).astype(np.uint32)
    seen[:5] = [1, 1, 1, 1, 3]                    # a count of 3 still penalises once
    for presence, repetition in [(0.0, 1.0), (0.5, 1.3), (2.0, 0.7), (-0.25, 1.1)]:
        got = orc.apply_penalties(logits, seen, presence, repetition)
        ref = _reference_loop(logits, seen, presence, repetition)
        assert np.array_equal(got.view(np.uint32), ref.view(np.uint32)), (presence, repetition)
    # the defaults leave every logit bit-identical
    assert np.array_equal(orc.apply_penalties(logits, seen, 0.0, 1.0).view(np.uint32), logits.view(np.uint32))


def test_mark_seen_counts_per_row_and_skips_out_of_range():
    seen = np.zeros((3, 10), np.uint32)
    orc.mark_seen(seen, [4, 4, -1])
    orc.mark_seen(seen, [4, 9, 10])
    assert seen[0, 4] == 2 and seen[1, 4] == 1 and seen[1, 9] == 1 and seen[2].sum() == 0
