"""Tensor parallelism on 2, 4 and 8 GPUs (one process per GPU, NCCL inside the
library): a TP model loaded from the same IMP-format export must produce the
oracle's greedy tokens and logits (within 1e-3 relative) for prefill + 24
decode steps, through both du_decode_step and the device-resident
du_decode_loop.  Each world size runs the decode reductions three ways:
ncclAllReduce only; the NVLink peer-memory allreduce fused into the O / down
GEMV epilogue (DU_TP_FUSE=1); and the same protocol as a separate kernel after
the GEMV (DU_TP_FUSE=0).  Cases with more ranks than GPUs are skipped.

The shapes keep every sharded K a whole, even number of INT4 groups up to 8
ranks: 16 q / 8 kv heads of 128, hidden 512, FFN 2048."""
import ctypes as C
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

CFG = dict(hidden=512, inter=2048, layers=2, hq=16, hkv=8, hd=128, vocab=2048)
MODES = {"nccl": (False, None), "p2p_fused": (True, "1"), "p2p_separate": (True, "0")}


def _rank(rank, world, q_in, q_out, q_h, p2p, fuse):
    try:
        if fuse is not None:     # read once per process by the library, so set it before the first call
            os.environ["DU_TP_FUSE"] = fuse
        torch.cuda.set_device(rank)
        from deepunity_b200 import _lib, LlamaForCausalLM, LLMQuant
        from tests.modelgen import ModelWeights, TestConfig
        cfg = TestConfig(**CFG, quant="int4", group=128)
        w = ModelWeights(cfg, seed=11)
        m = LlamaForCausalLM(cfg.du_kwargs(), LLMQuant.INT4, max_context_length=128, seed=None, device=rank,
                             tp_rank=rank, tp_size=world)
        w.load_into(m)
        if rank == 0:
            buf = C.create_string_buffer(128)
            _lib.call("du_nccl_unique_id", buf)
            for _ in range(world - 1):
                q_in.put(buf.raw)
            uid = buf.raw
        else:
            uid = q_in.get(timeout=120)
        m.init_tp(uid, timeout_ms=60000)
        if p2p:     # rank 0 gathers the IPC handles and hands every rank the full list
            if rank == 0:
                hs = {0: m.p2p_handle()}
                for _ in range(world - 1):
                    r_, h_ = q_h.get(timeout=120)
                    hs[r_] = h_
                allh = [hs[r_] for r_ in range(world)]
                for _ in range(world - 1):
                    q_in.put(allh)
            else:
                q_h.put((rank, m.p2p_handle()))
                allh = q_in.get(timeout=120)
            m.init_p2p(allh)
        prompt = np.random.default_rng(5).integers(0, cfg.vocab, 12).astype(np.int32)
        logits, nxt = m.forward(prompt[None, :])
        toks = [int(nxt[0])]
        for _ in range(11):
            toks.append(int(m.decode_step([toks[-1]])[0]))
        step_logits = m.read_logits(1)[0]
        toks += m.decode_loop([toks[-1]], 12)[:, 0].tolist()
        q_out.put((rank, logits[0], step_logits, toks))
        m.Release()
    except Exception as e:  # report to the parent instead of hanging it
        q_out.put((rank, None, None, repr(e)))


_REF = {}


def _oracle():
    if not _REF:
        from oracle import oracle as orc
        from tests.modelgen import ModelWeights, TestConfig
        cfg = TestConfig(**CFG, quant="int4", group=128)
        om = orc.OracleModel(ModelWeights(cfg, seed=11), capacity=128)
        prompt = np.random.default_rng(5).integers(0, cfg.vocab, 12).astype(np.int32)
        ref = om.forward(prompt)
        rt = [orc.argmax(ref)]
        for _ in range(11):
            last = om.forward([rt[-1]])
            rt.append(orc.argmax(last))
        ref_step = last
        for _ in range(12):
            rt.append(orc.argmax(om.forward([rt[-1]])))
        _REF.update(ref=ref, ref_step=ref_step, tokens=rt)
    return _REF


@pytest.mark.parametrize("mode", list(MODES))
@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_matches_oracle(world, mode):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    p2p, fuse = MODES[mode]
    ctx = mp.get_context("spawn")
    q_in, q_out, q_h = ctx.Queue(), ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, q_in, q_out, q_h, p2p, fuse)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, lg, slg, toks = q_out.get(timeout=600)
            res[r] = (lg, slg, toks)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert res[r][0] is not None, res[r][2]
    d = _oracle()
    for r in range(world):
        lg, slg, toks = res[r]
        assert float(np.max(np.abs(lg - d["ref"])) / np.max(np.abs(d["ref"]))) < 1e-3
        assert float(np.max(np.abs(slg - d["ref_step"])) / np.max(np.abs(d["ref_step"]))) < 1e-3
        assert toks == d["tokens"], (r, toks, d["tokens"])


def test_peer_wait_times_out_and_reports_it():
    """The bounded wait of the peer-memory reduction: rank 0 of a two-rank group whose
    rank 1 never writes must give up after the spin limit, set the error word the host
    reads, and leave the context usable (no rank, collective or kernel is left waiting)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from deepunity_b200 import _lib
    _lib.call("du_init", 0)
    flag = C.c_int(-1)
    _lib.call("du_tp_wait_selftest", 1 << 12, C.byref(flag))
    assert flag.value == 1
    # the context still works afterwards
    x = torch.arange(8, device="cuda", dtype=torch.float32)
    assert float(x.sum().item()) == 28.0
