"""Tensor-parallel host logic on CPU ranks (gloo, world size 2): the partition
the loader applies (du_tp_shard_window, the same function du_model_load_tensor
uses) tiles every tensor exactly, keeps whole heads and whole INT4 groups on a
rank, and the NCCL unique id reaches every rank intact."""
import ctypes as C
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from deepunity_b200 import _lib
from deepunity_b200.llm import CONFIGS

TENSORS = ["self_attn_q_proj", "self_attn_k_proj", "self_attn_v_proj", "self_attn_o_proj",
           "mlp_gate_proj", "mlp_up_proj", "mlp_down_proj", "lm_head"]


def cfg_for(name, tp, rank, quant=2, group=128):
    c = CONFIGS[name]
    m = _lib.ModelConfig()
    m.hidden_size, m.intermediate_size, m.num_layers = c.hidden_size, c.intermediate_size, c.num_layers
    m.num_heads_q, m.num_heads_kv, m.head_dim, m.vocab_size = c.num_heads_q, c.num_heads_kv, c.head_dim, c.vocab_size
    m.rms_eps, m.rope_theta, m.embed_scale = c.rms_eps, c.rope_theta, 1.0
    m.quant, m.group_size, m.kv_capacity, m.max_batch = quant, group, 8192, 1
    m.tp_rank, m.tp_size = rank, tp
    return m


def windows(name, tp, rank):
    out = {}
    for t in TENSORS:
        w = (C.c_int64 * 6)()
        _lib.call("du_tp_shard_window", C.byref(cfg_for(name, tp, rank)), t.encode(), w)
        out[t] = list(w)
    return out


def check_tiling(all_windows, name, tp):
    c = CONFIGS[name]
    for t in TENSORS:
        ws = [all_windows[r][t] for r in range(tp)]
        rows, cols = ws[0][0], ws[0][1]
        cover = np.zeros((rows, 1), np.int32) if all(w[4] == 0 and w[5] == cols for w in ws) else None
        if cover is not None:            # row split
            for w in ws:
                cover[w[2]:w[3]] += 1
                if t in ("self_attn_q_proj", "self_attn_k_proj", "self_attn_v_proj"):
                    assert w[2] % c.head_dim == 0 and w[3] % c.head_dim == 0, (t, w)
        else:                            # column split, every row kept
            cover = np.zeros((1, cols), np.int32)
            for w in ws:
                assert (w[2], w[3]) == (0, rows)
                cover[0, w[4]:w[5]] += 1
                assert w[4] % 128 == 0 and (w[5] - w[4]) % 256 == 0, (t, w)   # even number of int4 groups
        assert (cover == 1).all(), (name, tp, t)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = windows("llama-8b", world, rank)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        uid = [None]
        if rank == 0:
            buf = C.create_string_buffer(128)
            rc = _lib.lib().du_nccl_unique_id(buf)
            uid[0] = buf.raw if rc == 0 else b""
        dist.broadcast_object_list(uid, src=0)
        q.put((rank, gathered, uid[0]))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_two_rank_partition_and_unique_id_exchange():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort(key=lambda x: x[0])
    check_tiling(res[0][1], "llama-8b", 2)
    assert res[0][1] == res[1][1]
    uid0, uid1 = res[0][2], res[1][2]
    if uid0 == b"":
        pytest.skip("NCCL not loadable on this host")
    assert len(uid0) == 128 and uid0 == uid1


@pytest.mark.parametrize("name", ["llama-8b", "llama-1.1b"])
@pytest.mark.parametrize("tp", [1, 2, 4, 8])
def test_partition_tiles_every_tensor(name, tp):
    c = CONFIGS[name]
    if c.num_heads_kv % tp:
        pytest.skip("kv heads do not divide")
    group = 128 if name == "llama-8b" else 32
    try:
        all_w = [windows(name, tp, r) for r in range(tp)]
    except _lib.DUError:
        pytest.skip("configuration not valid at this tp degree")
    check_tiling(all_w, name, tp)


def test_partition_rejects_indivisible_degrees():
    with pytest.raises(_lib.DUError):
        windows("llama-8b", 3, 0)
