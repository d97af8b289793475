"""Tensor parallelism on 2 GPUs (one process per GPU, NCCL inside the library):
a TP=2 model loaded from the same IMP-format export must produce the oracle's
greedy tokens and logits (within 1e-3 relative) for prefill + 24 decode steps,
through both du_decode_step and the device-resident du_decode_loop, with the
decode reductions on NCCL and on the NVLink peer-memory allreduce
(du_tp_comm_open).  Skipped with fewer than 2 GPUs."""
import ctypes as C
import os

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

CFG = dict(hidden=512, inter=1024, layers=2, hq=8, hkv=4, hd=64, vocab=2048)


def _rank(rank, world, q_in, q_out, q_h, p2p):
    try:
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


@pytest.mark.parametrize("p2p", [False, True], ids=["nccl", "p2p"])
def test_tp2_matches_oracle(p2p):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    ctx = mp.get_context("spawn")
    q_in, q_out, q_h = ctx.Queue(), ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, q_in, q_out, q_h, p2p)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, lg, slg, toks = q_out.get(timeout=600)
        res[r] = (lg, slg, toks)
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert res[r][0] is not None, res[r][2]

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
    for r in range(2):
        lg, slg, toks = res[r]
        assert float(np.max(np.abs(lg - ref)) / np.max(np.abs(ref))) < 1e-3
        assert float(np.max(np.abs(slg - ref_step)) / np.max(np.abs(ref_step))) < 1e-3
        assert toks == rt, (r, toks, rt)
