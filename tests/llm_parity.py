"""Teacher-forced greedy parity of the LLM driver against the oracle decoder
(test infrastructure shared by tests/test_gpu_llm*.py and tests/tp_worker.py).

Protocol (the reference's decode loop, example/main_llm.cpp:622-654: logits of
the last position -> greedy_sample -> append -> repeat):
1. The GPU model runs prefill + `steps` greedy decode steps with logits
   requested (eager launches), recording logits and ids.
2. The same model runs again without logits: decode steps replay a CUDA graph
   and the LM head reduces straight to ids (fused argmax).  Those ids must
   equal run 1's bit for bit.
3. The oracle decoder (tests/llm_ref.py, KV-cached) follows the GPU's token
   sequence (teacher forcing) and produces its own logits per step.

Per step: logits rel-L2 and max-abs against the oracle within the stated
tolerance, and the GPU's id equal to the oracle's greedy id (the reference's
256-lane tie rule) unless the oracle's top-2 gap is at most 2 * max|dlogit|
of that step.  Within that bound a flip is arithmetically possible (each of
the two logits may move by the error); the step is then a "close call",
counted and reported with its gap.  Above it, any mismatch fails.
"""
import json
import os

import numpy as np

import oracle

# Stated logit tolerances against the oracle (rel-L2, max-abs excess over one
# storage ulp of the reference value).
LOGIT_TOL = {0: (5e-3, 2e-2), 1: (2e-2, 6e-2)}


def _host(t):
    import torch

    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def load_weights(model, ref, tdt):
    """Copies the oracle decoder's weights into an evk_b200.Llm (the driver
    slices them per tensor-parallel rank)."""
    import torch

    def dev(a):
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(tdt).cuda()

    model.set_weight("embedding", dev(ref.emb))
    if not ref.tied:
        model.set_weight("lm_head", dev(ref.lm_head))
    for l, w in enumerate(ref.w):
        for n in ("wqkv", "wo", "w1", "w2"):
            model.set_weight(n, dev(w[n]), layer=l)
    torch.cuda.synchronize()


def gpu_run(model, prompt, steps, V, tdt, with_logits):
    """prompt int32 [B, S] -> (ids [steps + 1, B], logits [steps + 1, B, V] or None)."""
    import torch

    B = prompt.shape[0]
    stream = torch.cuda.Stream()
    ids, logits = [], []
    with torch.cuda.stream(stream):
        tok = torch.from_numpy(np.ascontiguousarray(prompt, dtype=np.int32)).cuda()
        nxt = torch.zeros(B, dtype=torch.int32, device="cuda")
        lg = torch.empty(B, V, dtype=tdt, device="cuda") if with_logits else None
        model.prefill(tok, nxt, lg, stream=stream)
        ids.append(nxt.clone())
        if with_logits:
            logits.append(lg.clone())
        cur = nxt.clone()
        for _ in range(steps):
            out = torch.zeros(B, dtype=torch.int32, device="cuda")
            model.decode(cur, out, lg, stream=stream)
            ids.append(out)
            if with_logits:
                logits.append(lg.clone())
            cur = out
    torch.cuda.synchronize()
    idn = torch.stack(ids).cpu().numpy().astype(np.int64)
    lgn = np.stack([_host(x) for x in logits]) if with_logits else None
    return idn, lgn


def check_step(ref_logits, got_logits_u16, got_ids, dtype, stats, step):
    """One step's logits and ids against the oracle (see module docstring)."""
    B, V = ref_logits.shape
    r = oracle.to_float(ref_logits.ravel(), dtype).reshape(B, V).astype(np.float64)
    g = oracle.to_float(np.ascontiguousarray(got_logits_u16).ravel(), dtype).reshape(B, V).astype(np.float64)
    d = np.abs(g - r)
    err = d.max()
    rel = np.linalg.norm(g - r) / np.linalg.norm(r)
    rel_tol, abs_tol = LOGIT_TOL[dtype]
    ulp = (2.0 ** -10 if dtype == 0 else 2.0 ** -7) * np.abs(r)
    excess = (d - ulp).max()
    stats["max_rel_l2"] = max(stats.get("max_rel_l2", 0.0), float(rel))
    stats["max_abs"] = max(stats.get("max_abs", 0.0), float(err))
    assert rel <= rel_tol, f"step {step}: logits rel-L2 {rel:.3g} > {rel_tol}"
    assert excess <= abs_tol, f"step {step}: logits max-abs excess {excess:.3g} > {abs_tol}"
    rid = np.zeros(B, np.uint32)
    oracle.greedy_sample(np.ascontiguousarray(ref_logits).ravel(), rid, B, 1, V, 0, 0, V, dtype)
    bound = 2.0 * err
    for b in range(B):
        top2 = np.sort(r[b])[-2:]
        gap = float(top2[1] - top2[0])
        stats["checked"] += 1
        if gap <= bound:
            stats["near"] += 1  # a flip here is within the arithmetic error
        if int(got_ids[b]) != int(rid[b]):
            assert gap <= bound, (f"step {step} row {b}: greedy id {got_ids[b]} != oracle {rid[b]} with top-2 gap "
                                  f"{gap:.4g} > 2*max|dlogit| {bound:.4g}")
            stats["close_calls"].append({"step": step, "row": b, "gap": gap, "bound": float(bound)})
    return rid


def oracle_check(ref, prompt, ids, logits, dtype, max_len, tag):
    """Steps 3 and the per-step checks: the oracle follows `ids` (the GPU's
    greedy tokens) and every step's logits / ids are checked."""
    steps = ids.shape[0] - 1
    stats = {"config": tag, "checked": 0, "near": 0, "close_calls": []}
    rl = ref.start(prompt, max_len)
    rid = check_step(rl, logits[0], ids[0], dtype, stats, 0)
    equal = int(np.sum(rid == ids[0]))
    for s in range(1, steps + 1):
        rl = ref.step(ids[s - 1])  # the GPU's token: teacher forcing
        rid = check_step(rl, logits[s], ids[s], dtype, stats, s)
        equal += int(np.sum(rid == ids[s]))
    stats["fused_ids_equal_oracle"] = equal
    log = os.environ.get("EVKCU_PARITY_LOG")
    if log:
        with open(log, "a") as f:
            f.write(json.dumps(stats) + "\n")
    print(json.dumps(stats), flush=True)
    return stats


def teacher_forced_parity(ref, model, prompt, steps, dtype, tdt, max_len, tag):
    """Runs the protocol of the module docstring; returns the stats dict."""
    ids_l, logits = gpu_run(model, prompt, steps, ref.V, tdt, with_logits=True)
    ids_f, _ = gpu_run(model, prompt, steps, ref.V, tdt, with_logits=False)
    assert np.array_equal(ids_f, ids_l), "fused-argmax graph ids differ from the logits path"
    return oracle_check(ref, prompt, ids_f, logits, dtype, max_len, tag)
