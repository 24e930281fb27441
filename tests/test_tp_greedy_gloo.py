"""Vocabulary-sharded greedy sampling protocol on CPU ranks (gloo, world 2).

Each rank takes the 64-bit selection key of its vocabulary shard (global
token indices, as the driver's argmax_key_kernel does), the keys are
all-gathered and the maximum decoded: the result must equal the reference's
single-argmax tie rule (the oracle's literal 256-lane scan and tree) over the
whole vocabulary, including planted ties across shards.
"""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle

FMAX = np.finfo(np.float32).max


def bitrev8(x):
    return int(f"{x:08b}"[::-1], 2)


def key(v, j):
    if not (v > -FMAX):
        return 0
    if v == 0:
        v = 0.0  # -0.0 ties with +0.0, as `>` treats them
    u = np.float32(v).view(np.uint32).item()
    u = (~u & 0xFFFFFFFF) if (u & 0x80000000) else (u | 0x80000000)
    rank = (bitrev8(j & 255) << 24) | (j >> 8)
    return (u << 32) | (0xFFFFFFFF - rank)


def key_to_token(k):
    r = 0xFFFFFFFF - (k & 0xFFFFFFFF)
    return (r & 0xFFFFFF) * 256 + bitrev8(r >> 24)


def worker(rank, world, port, logits_f, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    V = logits_f.shape[1]
    Vl = V // world
    B = logits_f.shape[0]
    local = np.zeros(B, np.uint64)
    for b in range(B):
        best = 0
        for j in range(Vl):
            g = rank * Vl + j
            best = max(best, key(logits_f[b, g], g))
        local[b] = best
    gathered = [torch.zeros(B, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(gathered, torch.from_numpy(local.view(np.int64)))
    if rank == 0:
        keys = np.stack([g.numpy().view(np.uint64) for g in gathered])
        best = keys.max(axis=0)
        out.extend([int(key_to_token(int(k))) if k else 0 for k in best])
    dist.destroy_process_group()


@pytest.mark.parametrize("seed", [0, 1])
def test_sharded_greedy_matches_reference_rule(seed):
    rng = np.random.default_rng(seed)
    B, V = 4, 2048
    vals = rng.integers(-3, 3, size=(B, V)).astype(np.float32)
    vals[0, 5] = vals[0, 5 + 1024] = 9.0  # tie across the two shards
    vals[1, 300] = vals[1, 44] = 9.0      # tie inside shard 0, different lanes
    vals[3] = -1.0 - np.abs(vals[3])      # maximum 0 held by -0.0 (lane 3) and +0.0 (lane 7):
    vals[3, 3], vals[3, 7 + 1024] = -0.0, 0.0  # the lower bit-reversed lane (3) wins
    logits = oracle.from_float(vals.ravel())
    logits_f = oracle.to_float(logits).reshape(B, V)
    ref = np.zeros(B, np.uint32)
    oracle.greedy_sample(logits, ref, B, 1, V, 0, 0, V)
    with mp.Manager() as mgr:
        out = mgr.list()
        mp.spawn(worker, args=(2, 29600 + seed, logits_f, out), nprocs=2, join=True)
        got = list(out)
    assert got == ref.tolist()
