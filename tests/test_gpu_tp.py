"""Tensor parallelism on two GPUs: TP=2 against TP=1 on the same weights.

q/k/v/gate/up are column-split, o_proj/down_proj row-split with one NCCL
all-reduce each per layer, lm_head vocab-split with a gathered argmax that
keeps the last-index tie rule (engine.rs:256-261). In the exact numerics the
two layouts differ only in the order of the K sums split across ranks, so
logits agree to ~1e-5 and the greedy streams are identical. One process per
GPU (spawned), the NCCL id exchanged over a gloo group on 127.0.0.1. Needs
two GPUs; skipped otherwise.
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg():
    return dict(vocab_size=1000, hidden_size=512, num_layers=2, num_heads=8, num_kv_heads=2, head_dim=64,
                intermediate_size=1024, max_context=64, rope_theta=10000.0, rms_norm_eps=1e-5)


def _worker(rank, world, port, out_dir):
    import ctypes

    import torch
    import torch.distributed as dist

    import oracle as orc
    from golden_models import make_weights
    from beacon_cuda import CudaBackend, CudaModel, DecoderConfig
    from beacon_cuda import _lib as L

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    be = CudaBackend(rank, L.NUMERICS_EXACT)
    uid = torch.zeros(128, dtype=torch.uint8)
    if rank == 0:
        buf = (ctypes.c_uint8 * 128)()
        L.check(L.lib().beacon_cuda_comm_unique_id(buf))
        uid.copy_(torch.tensor(list(buf), dtype=torch.uint8))
    dist.broadcast(uid, 0)
    L.check(L.lib().beacon_cuda_comm_init(be.ctx, world, rank, (ctypes.c_uint8 * 128)(*uid.tolist()), 60000))
    c = _cfg()
    oc = orc.OracleModelConfig(**c)
    w = make_weights(oc, orc.Q4_K, seed=91)

    def build(tp, tr):
        m = CudaModel(be, DecoderConfig(**c, numerics=L.NUMERICS_EXACT, kv_dtype=L.DTYPE_F32, tp_size=tp, tp_rank=tr))
        for (layer, which), (data, dt) in w.items():
            m.set_weight(layer, which, data, dt)
        return m

    def run(m):
        prompt = [3, 14, 15, 92, 65, 35, 89, 79]
        logits = [m.forward(prompt, 0)[-1]]
        tok, toks, pos = int(np.argmax(logits[0])), [], len(prompt)
        for _ in range(8):
            nxt, lg = m.decode_step([tok], pos, want_logits=True)
            logits.append(lg[0])
            tok = int(nxt[0])
            toks.append(tok)
            pos += 1
        return np.stack(logits), toks

    m2 = build(world, rank)
    lg2, tk2 = run(m2)
    m2.close()
    if rank == 0:
        be1 = CudaBackend(rank, L.NUMERICS_EXACT)  # a context without a communicator
        w1 = CudaModel(be1, DecoderConfig(**c, numerics=L.NUMERICS_EXACT, kv_dtype=L.DTYPE_F32))
        for (layer, which), (data, dt) in w.items():
            w1.set_weight(layer, which, data, dt)
        lg1, tk1 = run(w1)
        w1.close()
        np.savez(os.path.join(out_dir, "tp.npz"), lg1=lg1, lg2=lg2, tk1=np.array(tk1), tk2=np.array(tk2))
    dist.barrier()
    be.close()
    dist.destroy_process_group()


def test_tp2_matches_tp1(tmp_path, cuda_lib):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    r = np.load(tmp_path / "tp.npz")
    assert np.abs(r["lg2"] - r["lg1"]).max() <= TOL * max(1.0, np.abs(r["lg1"]).max())
    assert r["tk2"].tolist() == r["tk1"].tolist()
