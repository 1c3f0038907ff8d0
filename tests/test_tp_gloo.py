"""The tensor-parallel sharding scheme on two CPU ranks (gloo), with the oracle
as the compute: what each GPU rank does, minus the GPU.

- column split (q/k/v/gate/up): rank r owns W rows [r N/2, (r+1) N/2) and its
  block bytes are a contiguous row slice; the gathered outputs equal the
  unsharded GEMV exactly (each row's sum is unchanged);
- row split (o_proj/down_proj): rank r owns K columns [r K/2, (r+1) K/2),
  whole super-blocks per row; rank 0 adds the residual to its partial and a
  sum all-reduce gives residual + W x (only the summation order changes);
- the vocab-split lm_head gathers [rank][rows][V/2] logits and the greedy
  pick over the concatenation keeps the last index of equal maxima
  (engine.rs:256-261), also when the tie straddles the shard boundary.
"""
import os
import socket

import numpy as np
import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rows(raw, dtype, n, k, r0, r1):
    import oracle as orc
    rb = (k // orc.block_size(dtype)) * orc.block_bytes(dtype)
    return raw.reshape(n, rb)[r0:r1].reshape(-1)


def _cols(raw, dtype, n, k, c0, c1):
    import oracle as orc
    bs, bb = orc.block_size(dtype), orc.block_bytes(dtype)
    blocks = raw.reshape(n, k // bs, bb)
    return np.ascontiguousarray(blocks[:, c0 // bs:c1 // bs]).reshape(-1)


def _worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist

    import oracle as orc

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    rng = np.random.default_rng(5)  # identical on every rank
    dtype, n, k = orc.Q4_K, 64, 1024
    raw = orc.quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32), dtype, orc.NIBBLE_REF_INTERLEAVED)
    x = rng.standard_normal((3, k)).astype(np.float32)
    res = rng.standard_normal((3, n)).astype(np.float32)
    full = orc.qgemv(raw, dtype, n, k, x)

    # column split
    r0, r1 = rank * n // world, (rank + 1) * n // world
    part = orc.qgemv(_rows(raw, dtype, n, k, r0, r1), dtype, r1 - r0, k, x)
    gathered = [torch.zeros(3, r1 - r0) for _ in range(world)]
    dist.all_gather(gathered, torch.from_numpy(np.ascontiguousarray(part)))
    col = torch.cat(gathered, dim=1).numpy()

    # row split with the residual added on rank 0
    c0, c1 = rank * k // world, (rank + 1) * k // world
    y = orc.qgemv(_cols(raw, dtype, n, k, c0, c1), dtype, n, c1 - c0, np.ascontiguousarray(x[:, c0:c1]))
    if rank == 0:
        y = y + res
    t = torch.from_numpy(np.ascontiguousarray(y))
    dist.all_reduce(t)
    row = t.numpy()

    # vocab split: a tie across the boundary and one inside rank 1's shard
    V = 100
    logits = rng.standard_normal((2, V)).astype(np.float32)
    logits[0, [10, 60]] = 9.0
    logits[1, [70, 71]] = 9.0
    shard = torch.from_numpy(np.ascontiguousarray(logits[:, rank * V // world:(rank + 1) * V // world]))
    parts = [torch.zeros_like(shard) for _ in range(world)]
    dist.all_gather(parts, shard)
    picks = [orc.argmax(r) for r in torch.cat(parts, dim=1).numpy()]
    if rank == 0:
        np.savez(os.path.join(out_dir, "tp.npz"), full=full, col=col, row=row, ref_row=full + res,
                 picks=np.array(picks), ref_picks=np.array([orc.argmax(r) for r in logits]))
    dist.barrier()
    dist.destroy_process_group()


def test_tp_sharding_scheme_on_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    r = np.load(tmp_path / "tp.npz")
    assert np.array_equal(r["col"], r["full"])                     # column split: bit-exact
    assert np.abs(r["row"] - r["ref_row"]).max() <= 1e-5 * np.abs(r["ref_row"]).max()
    assert r["picks"].tolist() == [60, 71] == r["ref_picks"].tolist()
