"""Whole-model parity on the GPU: the executor behind du_forward /
du_decode_step / du_decode_loop against the oracle's restatement of
MiniCPM5Model.Forward, on identical weights loaded from an IMP-format export.

Gates (north star): layer/logit outputs within max relative error 1e-3
(max|gpu - oracle| / max|oracle| over the logits), greedy token ids identical
for 64 steps."""
import numpy as np
import pytest
import torch

from deepunity_b200 import DUError, KVQuant, LlamaForCausalLM, LLMQuant, _lib
from oracle import oracle as orc
from tests.modelgen import C4, C5_SLICE, MID, SMALL, ModelWeights, TestConfig

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-3


@pytest.fixture(scope="module", autouse=True)
def device():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    yield


def relerr(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def build(cfg: TestConfig, seed=0, cap=128, max_batch=1, flags=0, kv_quant=KVQuant.FP16):
    w = ModelWeights(cfg, seed=seed)
    q = {"int8": LLMQuant.INT8, "int4": LLMQuant.INT4, "fp16": LLMQuant.FP16}[cfg.quant]
    m = LlamaForCausalLM(cfg.du_kwargs(), q, kv_quant=kv_quant, max_context_length=cap, max_batch=max_batch, seed=None,
                         flags=flags)
    w.load_into(m)
    return w, m


# decode steps: the persistent decode-step kernel (default) and the graph of per-stage kernels
PATHS = {"persistent": _lib.FLAG_PERSISTENT, "per_stage": 0}


VARIANTS = [SMALL, MID,
            TestConfig(256, 512, 2, 4, 2, 64, 1024, quant="int4", group=128),
            TestConfig(512, 1024, 2, 4, 1, 128, 2048, quant="int4", group=32),
            TestConfig(256, 512, 2, 4, 4, 64, 1024, quant="fp16")]


@pytest.mark.parametrize("path", list(PATHS))
@pytest.mark.parametrize("cfg", VARIANTS, ids=lambda c: f"{c.quant}-h{c.hidden}-hd{c.hd}-g{c.group}")
def test_prefill_then_greedy_64_matches_oracle(cfg, path):
    w, m = build(cfg, cap=128, flags=PATHS[path])
    om = orc.OracleModel(w, capacity=128)
    prompt = np.random.default_rng(7).integers(0, cfg.vocab, 16).astype(np.int32)
    logits, nxt = m.forward(prompt[None, :])
    ref = om.forward(prompt)
    assert relerr(logits[0], ref) < LOGIT_TOL
    assert int(nxt[0]) == orc.argmax(ref)
    toks, rtoks = [int(nxt[0])], [orc.argmax(ref)]
    for _ in range(63):
        toks.append(int(m.decode_step([toks[-1]])[0]))
        r = om.forward([rtoks[-1]])
        rtoks.append(orc.argmax(r))
    assert toks == rtoks
    assert relerr(m.read_logits(1)[0], r) < LOGIT_TOL
    assert m.cache_len() == 16 + 63
    m.Release()
    m.Release()   # idempotent


def test_predict_all_positions_and_device_loop():
    """Stateless Predict over 20 positions (the lm_head of all positions runs as the
    tensor-core GEMM with its logits + argmax epilogue), then the device-resident loop."""
    cfg = MID
    w, m = build(cfg, cap=96)
    om = orc.OracleModel(w, capacity=96)
    prompt = np.random.default_rng(8).integers(0, cfg.vocab, 20).astype(np.int32)
    lg = m.Predict(prompt)
    ref = om.forward(prompt, last_pos_only=False)
    assert lg.shape == ref.shape
    assert relerr(lg, ref) < LOGIT_TOL
    # device-resident greedy loop == step-by-step oracle
    m.ResetCache()
    om.reset()
    _, nxt = m.forward(prompt[None, :])
    toks = m.decode_loop([int(nxt[0])], 40)[:, 0].tolist()
    r = om.forward(prompt)
    rt = [orc.argmax(r)]
    for _ in range(40):
        rt.append(orc.argmax(om.forward([rt[-1]])))
    assert [int(nxt[0])] + toks == rt
    m.Release()


def test_batched_sequences_match_independent_oracles():
    cfg = SMALL
    w, m = build(cfg, cap=96, max_batch=3)
    prompts = np.random.default_rng(9).integers(0, cfg.vocab, (3, 10)).astype(np.int32)
    logits, nxt = m.forward(prompts)
    oms = [orc.OracleModel(w, capacity=96) for _ in range(3)]
    refs = [om.forward(prompts[b]) for b, om in enumerate(oms)]
    for b in range(3):
        assert relerr(logits[b], refs[b]) < LOGIT_TOL
    cur = nxt.copy()
    rcur = [orc.argmax(r) for r in refs]
    assert cur.tolist() == rcur
    for _ in range(20):
        cur = m.decode_step(cur)
        rcur = [orc.argmax(om.forward([t])) for om, t in zip(oms, rcur)]
        assert cur.tolist() == rcur
    m.Release()


def test_errors_are_reported_not_crashed():
    cfg = SMALL
    w, m = build(cfg, cap=20)
    with pytest.raises(DUError):
        m.forward(np.array([[cfg.vocab]], np.int32))          # id out of range
    with pytest.raises(DUError):
        m.forward(np.zeros((1, 21), np.int32))                # beyond capacity
    with pytest.raises(DUError):
        m.load_tensor("layer_0/self_attn_q_proj.int8.bin", np.zeros(7, np.uint8))   # wrong size
    with pytest.raises(DUError):
        m.load_tensor("layer_9/self_attn_q_proj.int8.bin", np.zeros(7, np.uint8))   # unknown layer
    m.forward(np.zeros((1, 19), np.int32))
    m.decode_step([1])
    with pytest.raises(DUError):
        m.decode_step([1])                                    # cache full
    m.Release()


def test_config4_llama_1p1b_int8_greedy_64():
    """1.1B llama, INT8 per-row, 128-token random prompt, 64 greedy steps."""
    w, m = build(C4, seed=0, cap=256)
    om = orc.OracleModel(w, capacity=256)
    prompt = np.random.default_rng(0).integers(0, C4.vocab, 128).astype(np.int32)
    logits, nxt = m.forward(prompt[None, :])
    ref = om.forward(prompt)
    assert relerr(logits[0], ref) < LOGIT_TOL
    toks = [int(nxt[0])] + m.decode_loop([int(nxt[0])], 63)[:, 0].tolist()
    rt = [orc.argmax(ref)]
    for _ in range(63):
        rt.append(orc.argmax(om.forward([rt[-1]])))
    assert toks == rt
    m.Release()


# ---------------------------------------------------------------- BASELINE config 5
# The benchmarked 8B INT4-G128 architecture (hidden 4096, FFN 14336, 32 q / 8 kv
# heads of 128, vocab 128256) on a 2-layer slice: a 128-token prompt, then 64
# greedy ids.  The oracle run is shared by both decode paths.
_C5 = {}


def _c5_oracle():
    if not _C5:
        w = ModelWeights(C5_SLICE, seed=5)
        om = orc.OracleModel(w, capacity=256)
        prompt = np.random.default_rng(5).integers(0, C5_SLICE.vocab, 128).astype(np.int32)
        ref = om.forward(prompt)
        rt, last = [orc.argmax(ref)], None
        for _ in range(63):
            last = om.forward([rt[-1]])
            rt.append(orc.argmax(last))
        _C5.update(w=w, prompt=prompt, ref=ref, tokens=rt, last=last)
    return _C5


@pytest.mark.parametrize("path", list(PATHS))
def test_config5_slice_int4_g128_greedy_64(path):
    d = _c5_oracle()
    m = LlamaForCausalLM(C5_SLICE.du_kwargs(), LLMQuant.INT4, max_context_length=256, seed=None,
                         flags=PATHS[path])
    d["w"].load_into(m)
    logits, nxt = m.forward(d["prompt"][None, :])
    assert relerr(logits[0], d["ref"]) < LOGIT_TOL
    toks = [int(nxt[0])] + m.decode_loop([int(nxt[0])], 63)[:, 0].tolist()
    assert toks == d["tokens"]
    assert relerr(m.read_logits(1)[0], d["last"]) < LOGIT_TOL
    m.Release()


def test_config4_batch16_int8():
    """BASELINE config 4 at batch 16: 16 sequences prefilled and decoded together;
    the first, a middle and the last sequence are checked against independent
    oracle runs (logits of the prompt and 25 greedy ids)."""
    w, m = build(C4, seed=1, cap=64, max_batch=16)
    prompts = np.random.default_rng(16).integers(0, C4.vocab, (16, 16)).astype(np.int32)
    logits, nxt = m.forward(prompts)
    toks = m.decode_loop(nxt, 24)
    for b in (0, 7, 15):
        om = orc.OracleModel(w, capacity=64)
        ref = om.forward(prompts[b])
        assert relerr(logits[b], ref) < LOGIT_TOL, b
        rt = [orc.argmax(ref)]
        for _ in range(24):
            rt.append(orc.argmax(om.forward([rt[-1]])))
        assert [int(nxt[b])] + toks[:, b].tolist() == rt, b
    m.Release()


def _tree_rank(i: int):
    """Order of the reference ArgMax tree among tied maxima (G3CS:911-928):
    bit-reversed thread id (i % 256), then the lowest index of that thread."""
    t = i % 256
    return (int(f"{t:08b}"[::-1], 2), i // 256)


@pytest.mark.parametrize("path", list(PATHS))
def test_greedy_ties_follow_the_reference_argmax_tree(path):
    """Two lm_head rows made identical give bit-identical logits; the greedy pick must
    be the one the reference's ArgMax tree keeps, which here is not the lower index."""
    cfg = SMALL
    w = ModelWeights(cfg, seed=4)
    prompt = np.arange(3, 11, dtype=np.int32)
    top = orc.argmax(orc.OracleModel(w, capacity=64).forward(prompt))
    cands = [j for j in range(cfg.vocab) if j != top and (j < top) != (_tree_rank(j) < _tree_rank(top))]
    assert cands, top
    j = cands[0]
    w.lm_head[j] = w.lm_head[top]
    expect = top if _tree_rank(top) < _tree_rank(j) else j
    ref = orc.OracleModel(w, capacity=64).forward(prompt)
    assert ref[top] == ref[j] and orc.argmax(ref) == expect
    q = {"int8": LLMQuant.INT8, "int4": LLMQuant.INT4, "fp16": LLMQuant.FP16}[cfg.quant]
    m = LlamaForCausalLM(cfg.du_kwargs(), q, max_context_length=64, seed=None, flags=PATHS[path])
    w.load_into(m)
    logits, nxt = m.forward(prompt[None, :])
    assert logits[0][top] == logits[0][j]
    assert int(nxt[0]) == expect                       # prefill head + greedy pick
    m.ResetCache()
    m.forward(prompt[None, :-1])
    assert int(m.decode_step([prompt[-1]])[0]) == expect   # decode graph's head + pick
    m.Release()


@pytest.mark.parametrize("setting", [(0.8, 40, 0.9, 0.0), (1.0, 0, 1.0, 0.05), (0.0, 0, 1.0, 0.0)])
def test_sampled_decode_matches_oracle(setting):
    """du_decode_step_sample (SampleYielding, M5M:653-705): 16 sampled steps with a seed per
    step; each step's id must be what the oracle sampler draws from the oracle's logits."""
    T, k, p, mp = setting
    cfg = MID
    w, m = build(cfg, cap=96)
    om = orc.OracleModel(w, capacity=96)
    prompt = np.random.default_rng(12).integers(0, cfg.vocab, 10).astype(np.int32)
    logits, _ = m.forward(prompt[None, :])
    ref = om.forward(prompt)
    rng = np.random.default_rng(99)
    seed = int(rng.integers(-2 ** 31, 2 ** 31 - 1))
    tok = orc.sample(ref, T, k, p, mp, seed)
    toks, rtoks = [tok], [tok]
    for _ in range(16):
        seed = int(rng.integers(-2 ** 31, 2 ** 31 - 1))
        toks.append(int(m.decode_step_sample([toks[-1]], T, k, p, mp, [seed])[0]))
        rtoks.append(orc.sample(om.forward([rtoks[-1]]), T, k, p, mp, seed))
    assert toks == rtoks
    m.Release()


@pytest.mark.parametrize("setting", [(0.0, 0, 1.0, 0.0, 0.4, 1.3), (0.8, 40, 0.9, 0.0, 0.5, 1.2)])
def test_penalized_sampled_decode_matches_oracle(setting):
    """du_decode_step_sample_ex (DispatchSampleKernels, Qwen3_5Model.cs:1010-1058): the
    first id is picked from the prefill logits with nothing seen, then 16 steps whose
    input ids (the previous picks) count as seen; each step's id must be what the oracle
    picks after applying the same penalties to its logits.  ResetCache clears the counts:
    the first step after it sees only its own input."""
    T, k, p, mp, pres, rep = setting
    cfg = MID
    w, m = build(cfg, cap=96)
    om = orc.OracleModel(w, capacity=96)
    prompt = np.random.default_rng(13).integers(0, cfg.vocab, 10).astype(np.int32)
    m.forward(prompt[None, :])
    ref = om.forward(prompt)
    rng = np.random.default_rng(7)
    seed = int(rng.integers(-2 ** 31, 2 ** 31 - 1))
    tok = orc.sample(ref, T, k, p, mp, seed)
    toks, rtoks = [tok], [tok]
    seen = np.zeros((1, cfg.vocab), np.uint32)
    for _ in range(16):
        seed = int(rng.integers(-2 ** 31, 2 ** 31 - 1))
        toks.append(int(m.decode_step_sample_ex([toks[-1]], T, k, p, mp, pres, rep, [seed])[0]))
        orc.mark_seen(seen, [rtoks[-1]])
        r = orc.apply_penalties(om.forward([rtoks[-1]]), seen[0], pres, rep)
        rtoks.append(orc.sample(r, T, k, p, mp, seed))
    assert toks == rtoks
    assert len(set(toks)) > 1
    # after a cache reset only the new step's input is seen
    m.ResetCache()
    om.reset()
    m.forward(prompt[None, :])
    om.forward(prompt)
    seed = int(rng.integers(-2 ** 31, 2 ** 31 - 1))
    got = int(m.decode_step_sample_ex([toks[3]], T, k, p, mp, pres, rep, [seed])[0])
    fresh = np.zeros(cfg.vocab, np.uint32)
    fresh[toks[3]] = 1
    want = orc.sample(orc.apply_penalties(om.forward([toks[3]]), fresh, pres, rep), T, k, p, mp, seed)
    assert got == want
    m.Release()


KV8_LOGIT_TOL = 5e-3


def _near_tie(logits, tol=2e-3):
    """The two largest logits lie within tol * max|logit| of each other."""
    top = np.sort(logits)[-2:]
    return float(top[1] - top[0]) <= tol * float(np.max(np.abs(logits)))


@pytest.mark.parametrize("cfg", [SMALL, TestConfig(256, 512, 2, 4, 2, 128, 1024, quant="int4", group=128)],
                         ids=lambda c: f"{c.quant}-hd{c.hd}")
def test_int8_kv_cache_teacher_forced_64_matches_oracle(cfg):
    """KVQuant.INT8 (WriteCacheFull KV_INT8 + KV_READ_K / KV_READ_V): a 24-token prefill then
    64 teacher-forced decode steps (both sides are fed the oracle's greedy ids).  Every
    step's logits within 5e-3 and the greedy id equal unless the oracle's top two logits
    are a near-tie.  The 8-bit quantizer rounds each K / V value to its row's step
    (range / 255); fp32 values that differ by an ulp can round to neighbouring bytes, so
    the two caches may differ by one step in a few elements: that widens the logit gate
    from 1e-3 and makes free-running greedy comparisons flip at near-ties."""
    w, m = build(cfg, cap=128, kv_quant=KVQuant.INT8)
    om = orc.OracleModel(w, capacity=128, kv_int8=True)
    prompt = np.random.default_rng(11).integers(0, cfg.vocab, 24).astype(np.int32)
    logits, nxt = m.forward(prompt[None, :])
    ref = om.forward(prompt)
    assert relerr(logits[0], ref) < KV8_LOGIT_TOL
    tok = orc.argmax(ref)
    assert int(nxt[0]) == tok or _near_tie(ref)
    for step in range(64):
        got_id = int(m.decode_step([tok])[0])
        r = om.forward([tok])
        assert relerr(m.read_logits(1)[0], r) < KV8_LOGIT_TOL, step
        tok = orc.argmax(r)
        assert got_id == tok or _near_tie(r), step
    assert m.cache_len() == 24 + 64
    m.Release()


def test_int8_kv_cache_batched():
    """Three sequences decoding together over the INT8 cache, teacher-forced, each against
    its own oracle."""
    cfg = SMALL
    w, m = build(cfg, cap=96, max_batch=3, kv_quant=KVQuant.INT8)
    prompts = np.random.default_rng(12).integers(0, cfg.vocab, (3, 10)).astype(np.int32)
    logits, nxt = m.forward(prompts)
    oms = [orc.OracleModel(w, capacity=96, kv_int8=True) for _ in range(3)]
    refs = [oms[i].forward(prompts[i]) for i in range(3)]
    for i in range(3):
        assert relerr(logits[i], refs[i]) < KV8_LOGIT_TOL
    cur = [orc.argmax(r) for r in refs]
    for step in range(24):
        got = m.decode_step(cur)
        lg = m.read_logits(3)
        refs = [oms[i].forward([cur[i]]) for i in range(3)]
        for i in range(3):
            assert relerr(lg[i], refs[i]) < KV8_LOGIT_TOL, (step, i)
            assert int(got[i]) == orc.argmax(refs[i]) or _near_tie(refs[i]), (step, i)
        cur = [orc.argmax(r) for r in refs]
    m.Release()


# Gemma3 variants on the same kernels (Gemma3Model.cs:315-590): qk-norm, sandwich norms,
# GELU GLU, sqrt(H) embedding scale, sliding-window layers (every 3rd layer full) with
# their own RoPE base, a softmax scale of their own
GEMMA_VARIANTS = [
    TestConfig(256, 512, 3, 4, 1, 128, 1024, quant="int8", theta=1_000_000.0, arch=7, window=16, pattern=3,
               theta_local=10000.0, attn_scale=0.1, embed_scale=16.0, eps=1e-6),
    TestConfig(512, 1024, 3, 2, 1, 256, 1024, quant="int4", group=128, theta=1_000_000.0, arch=7, window=20,
               pattern=3, theta_local=10000.0, attn_scale=256 ** -0.5, embed_scale=512 ** 0.5, eps=1e-6),
]


@pytest.mark.parametrize("cfg", GEMMA_VARIANTS, ids=lambda c: f"{c.quant}-hd{c.hd}")
def test_gemma3_variant_greedy_64_matches_oracle(cfg):
    """A 24-token prompt then 64 greedy steps: positions run well past the sliding window,
    so the sliding-window layers attend to a moving band and the full layers to all."""
    w, m = build(cfg, cap=128)
    om = orc.OracleModel(w, capacity=128)
    prompt = np.random.default_rng(13).integers(0, cfg.vocab, 24).astype(np.int32)
    logits, nxt = m.forward(prompt[None, :])
    ref = om.forward(prompt)
    assert relerr(logits[0], ref) < LOGIT_TOL
    toks, rtoks = [int(nxt[0])], [orc.argmax(ref)]
    for _ in range(63):
        toks.append(int(m.decode_step([toks[-1]])[0]))
        r = om.forward([rtoks[-1]])
        rtoks.append(orc.argmax(r))
    assert toks == rtoks
    assert relerr(m.read_logits(1)[0], r) < LOGIT_TOL
    m.Release()


# Qwen3.5 full-attention layers on the same kernels (Qwen3_5Model.cs:397-574): q projection
# with a per-head output gate, qk-norm, partial RoPE over the first rot dims, attention output
# times sigmoid(gate) before o_proj
QWEN35_VARIANTS = [
    TestConfig(512, 1024, 3, 4, 1, 256, 1024, quant="int4", group=128, theta=10_000_000.0, arch=9, rot=64, eps=1e-6),
    TestConfig(256, 512, 2, 4, 2, 128, 1024, quant="int8", arch=9, rot=32, eps=1e-6),
]


@pytest.mark.parametrize("cfg", QWEN35_VARIANTS, ids=lambda c: f"{c.quant}-hd{c.hd}-rot{c.rot}")
def test_qwen35_full_attention_greedy_64_matches_oracle(cfg):
    """A 24-token prompt then 64 greedy steps: identical ids and final logits within 1e-3 of
    the oracle's restatement of QProjGated, RmsNormHead, ApplyRopePartial and ApplyAttnGate."""
    w, m = build(cfg, cap=128)
    om = orc.OracleModel(w, capacity=128)
    prompt = np.random.default_rng(17).integers(0, cfg.vocab, 24).astype(np.int32)
    logits, nxt = m.forward(prompt[None, :])
    ref = om.forward(prompt)
    assert relerr(logits[0], ref) < LOGIT_TOL
    toks, rtoks = [int(nxt[0])], [orc.argmax(ref)]
    for _ in range(63):
        toks.append(int(m.decode_step([toks[-1]])[0]))
        r = om.forward([rtoks[-1]])
        rtoks.append(orc.argmax(r))
    assert toks == rtoks
    assert relerr(m.read_logits(1)[0], r) < LOGIT_TOL
    m.Release()


def test_gemma3_variant_int8_kv_teacher_forced():
    """The Gemma3 variant over the INT8 cache (the qkv-post kernel quantizes k / v rows)."""
    cfg = GEMMA_VARIANTS[0]
    w, m = build(cfg, cap=128, kv_quant=KVQuant.INT8)
    om = orc.OracleModel(w, capacity=128, kv_int8=True)
    prompt = np.random.default_rng(14).integers(0, cfg.vocab, 24).astype(np.int32)
    logits, nxt = m.forward(prompt[None, :])
    ref = om.forward(prompt)
    assert relerr(logits[0], ref) < KV8_LOGIT_TOL
    tok = orc.argmax(ref)
    for step in range(48):
        got_id = int(m.decode_step([tok])[0])
        r = om.forward([tok])
        assert relerr(m.read_logits(1)[0], r) < KV8_LOGIT_TOL, step
        tok = orc.argmax(r)
        assert got_id == tok or _near_tie(r), step
    m.Release()


def test_fused_attention_o_matches_separate_o(monkeypatch):
    """One-row decode steps run the O projection inside the flash-decode kernel (W_o rows
    bulk-copied during attention, per-kv-head partial sums added in kv head order).  The
    same model with DU_FUSE_ATTN_O=0 runs a separate O GEMV: logits agree to 1e-5 and the
    greedy ids are identical; both match the oracle."""
    cfg = MID
    runs = {}
    for fuse in ("1", "0"):
        monkeypatch.setenv("DU_FUSE_ATTN_O", fuse)
        w, m = build(cfg, cap=96)
        prompt = np.random.default_rng(15).integers(0, cfg.vocab, 16).astype(np.int32)
        _, nxt = m.forward(prompt[None, :])
        toks, lg = [int(nxt[0])], []
        for _ in range(32):
            toks.append(int(m.decode_step([toks[-1]])[0]))
            lg.append(m.read_logits(1)[0].copy())
        runs[fuse] = (toks, np.stack(lg))
        m.Release()
    assert runs["1"][0] == runs["0"][0]
    assert relerr(runs["1"][1], runs["0"][1]) < 1e-5
    om = orc.OracleModel(w, capacity=96)
    ref = om.forward(prompt)
    rt = [orc.argmax(ref)]
    for _ in range(32):
        rt.append(orc.argmax(om.forward([rt[-1]])))
    assert runs["1"][0] == rt
