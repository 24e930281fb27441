"""Worker for tests/test_gpu_llm_tp.py (run under torchrun, one rank per GPU).

Every rank builds the same oracle-seeded decoder (tests/llm_ref.py weights,
sliced per rank by evkcu_llm_set_weight) with tensor parallelism over all
ranks (NCCL communicator from evkcu_comm_*, its id broadcast with
torch.distributed).  All ranks run prefill + decode twice: with logits (the
vocab-sharded logits all-gathered) and without (fused LM-head argmax per
shard, 64-bit keys all-gathered, CUDA-graph decode).  Rank 0 then checks the
ids and logits against the oracle decoder, teacher-forced on the GPU's
tokens (tests/llm_parity.py: ids bit-exact outside the arithmetic-error gap
bound).  Every rank checks the device error word (a timed-out fused
all-reduce is reported only there).  Prints TP_OK on success.
"""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)
import evk_b200 as ev  # noqa: E402
from llm_parity import gpu_run, load_weights, oracle_check  # noqa: E402
from llm_ref import RefModel  # noqa: E402

CFG = dict(layers=2, d_model=512, heads=8, hidden=2048, vocab=1024)
B, S, STEPS, MAX_SEQ = 2, 20, 6, 64


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
    tdt = torch.bfloat16
    prompt = np.random.default_rng(4).integers(0, CFG["vocab"], size=(B, S))
    for tied in (True, False):
        ref = RefModel(CFG["layers"], CFG["d_model"], CFG["heads"], CFG["hidden"], CFG["vocab"], tied, dtype=1,
                       seed=77)
        tp = ev.Llm(**CFG, max_batch=B, max_seq=MAX_SEQ, dtype=ev.BF16, tied_embeddings=tied, tp_rank=rank,
                    tp_size=world, comm=comm)
        load_weights(tp, ref, tdt)
        ids_l, logits = gpu_run(tp, prompt, STEPS, CFG["vocab"], tdt, with_logits=True)
        ids_f, _ = gpu_run(tp, prompt, STEPS, CFG["vocab"], tdt, with_logits=False)
        ev.check_device_error()
        tp.close()
        assert np.array_equal(ids_f, ids_l), (ids_f, ids_l)
        if rank == 0:
            oracle_check(ref, prompt, ids_f, logits, 1, MAX_SEQ, f"tp={world} tied={tied}")
    # The ranks agree on the decode all-reduce path: switching the fused one
    # off on one rank only makes every rank use NCCL (and decode runs to the
    # end instead of one rank waiting for peers that never arrive).
    ref = RefModel(CFG["layers"], CFG["d_model"], CFG["heads"], CFG["hidden"], CFG["vocab"], True, dtype=1, seed=77)
    paths = {}
    for one_off in (False, True):
        if one_off and rank == world - 1:
            os.environ["EVKCU_DISABLE_FUSED_ALLREDUCE"] = "1"
        tp = ev.Llm(**CFG, max_batch=B, max_seq=MAX_SEQ, dtype=ev.BF16, tied_embeddings=True, tp_rank=rank,
                    tp_size=world, comm=comm)
        os.environ.pop("EVKCU_DISABLE_FUSED_ALLREDUCE", None)
        load_weights(tp, ref, tdt)
        ids, _ = gpu_run(tp, prompt, 3, CFG["vocab"], tdt, with_logits=False)
        ev.check_device_error()
        flags = [None] * world
        dist.all_gather_object(flags, (tp.fused_allreduce, ids.tolist()))
        tp.close()
        assert all(f == flags[0] for f in flags), flags
        paths[one_off] = flags[0]
    assert paths[True][0] is False, "one rank without the fused path: all ranks use NCCL"
    if rank == 0:
        print(f"fused all-reduce: on everywhere -> {paths[False][0]}, off on one rank -> {paths[True][0]}",
              flush=True)
    dist.barrier()
    comm.close()
    dist.destroy_process_group()
    if rank == 0:
        print("TP_OK", flush=True)


if __name__ == "__main__":
    main()
