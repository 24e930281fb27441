"""Worker for tests/test_gpu_llm_tp.py (run under torchrun, one rank per GPU).

Every rank builds the same seeded decoder with tensor parallelism over all
ranks (NCCL communicator from evkcu_comm_*, its id broadcast with
torch.distributed); rank 0 also builds the single-GPU model and compares
prefill / decode logits and greedy ids.  Prints TP_OK on success.
"""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import evk_b200 as ev  # noqa: E402

CFG = dict(layers=2, d_model=512, heads=8, hidden=2048, vocab=1024, max_batch=2, max_seq=64)


def run(model, tokens, steps, V, tdt):
    B = tokens.shape[0]
    nxt = torch.zeros(B, dtype=torch.int32, device="cuda")
    lg = torch.empty(B, V, dtype=tdt, device="cuda")
    stream = torch.cuda.current_stream()
    model.prefill(tokens, nxt, lg, stream=stream)
    logits, ids = [lg.float().cpu()], [nxt.cpu()]
    cur = nxt.clone()
    for _ in range(steps):
        out = torch.zeros(B, dtype=torch.int32, device="cuda")
        model.decode(cur, out, lg, stream=stream)
        logits.append(lg.float().cpu())
        ids.append(out.cpu())
        cur = out
    torch.cuda.synchronize()
    return torch.stack(logits), torch.stack(ids)


def run_ids(model, tokens, steps):
    """Without logits: fused LM-head argmax (rank keys + all-gather), decode
    steps replayed as CUDA graphs."""
    B = tokens.shape[0]
    stream = torch.cuda.Stream()
    ids = []
    with torch.cuda.stream(stream):
        nxt = torch.zeros(B, dtype=torch.int32, device="cuda")
        model.prefill(tokens, nxt, stream=stream)
        ids.append(nxt.clone())
        cur = nxt.clone()
        for _ in range(steps):
            out = torch.zeros(B, dtype=torch.int32, device="cuda")
            model.decode(cur, out, stream=stream)
            ids.append(out)
            cur = out
    torch.cuda.synchronize()
    return torch.stack(ids).cpu()


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", device_id=torch.device("cuda", int(os.environ["LOCAL_RANK"])))
    ev.init(int(os.environ["LOCAL_RANK"]))
    uid = torch.zeros(128, dtype=torch.uint8, device="cuda")
    if rank == 0:
        uid.copy_(torch.frombuffer(bytearray(ev.Comm.unique_id()), dtype=torch.uint8))
    dist.broadcast(uid, 0)
    comm = ev.Comm(bytes(uid.cpu().numpy()), rank, world)
    dtype = ev.BF16
    tdt = torch.bfloat16
    tokens = torch.from_numpy(np.random.default_rng(4).integers(0, CFG["vocab"], size=(2, 20)).astype(np.int32)).cuda()
    for tied in (True, False):
        tp = ev.Llm(**CFG, dtype=dtype, tied_embeddings=tied, tp_rank=rank, tp_size=world, comm=comm)
        tp.init_random(seed=77, std=0.02)
        lt, it = run(tp, tokens, 6, CFG["vocab"], tdt)
        tp.close()
        # Same model again without logits: the fused head must pick the same ids.
        tp = ev.Llm(**CFG, dtype=dtype, tied_embeddings=tied, tp_rank=rank, tp_size=world, comm=comm)
        tp.init_random(seed=77, std=0.02)
        it_fused = run_ids(tp, tokens, 6)
        tp.close()
        assert torch.equal(it_fused, it), (it_fused, it)
        if rank == 0:
            one = ev.Llm(**CFG, dtype=dtype, tied_embeddings=tied)
            one.init_random(seed=77, std=0.02)
            l1, i1 = run(one, tokens, 6, CFG["vocab"], tdt)
            one.close()
            rel = ((lt - l1).norm() / l1.norm()).item()
            same = (it == i1).float().mean().item()
            print(f"tied={tied} logits rel-L2 {rel:.3g}, id agreement {same:.3f}", flush=True)
            assert rel < 2e-2, rel
            assert same >= 0.9, (it, i1)
    dist.barrier()
    comm.close()
    dist.destroy_process_group()
    if rank == 0:
        print("TP_OK", flush=True)


if __name__ == "__main__":
    main()
