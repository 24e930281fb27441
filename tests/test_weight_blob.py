"""Weight-blob format (evkcu_llm_load / evkcu_llm_save, include/evkcu.h):
the Python writer's layout on CPU, and on the GPU a model loaded from a blob
produces the same logits as one given the weights through set_weight, and
save -> load round-trips every weight."""
import os

import numpy as np
import pytest

import oracle
from conftest import has_gpu


def test_blob_layout_and_header_on_cpu(tmp_path):
    import evk_b200

    L, D, H, F, V = 2, 64, 4, 128, 300
    lay = evk_b200.blob_layout(L, D, H, F, V, tied_embeddings=False)
    assert [n for n, _, _ in lay[:3]] == ["embedding", "lm_head", "wqkv"]
    w = {(n, l): oracle.normal(s[0] * s[1], 3 + i) for i, (n, l, s) in enumerate(lay)}
    p = tmp_path / "m.evkw"
    evk_b200.write_weight_blob(p, w, L, D, H, F, V, tied_embeddings=False, dtype=evk_b200.BF16)
    raw = np.fromfile(p, np.uint8)
    hdr = raw[:64].view(np.uint32)
    assert raw[:8].tobytes() == b"EVKWBLOB"
    assert list(hdr[2:11]) == [1, 1, L, D, H, H, F, V, 0]
    body = raw[64:].view(np.uint16)
    off = 0
    for n, l, s in lay:
        cnt = s[0] * s[1]
        assert np.array_equal(body[off:off + cnt], w[(n, l)]), n
        off += cnt
    assert off == body.size
    with pytest.raises(ValueError):
        w[("w1", 1)] = w[("w1", 1)][:-1]
        evk_b200.write_weight_blob(tmp_path / "bad.evkw", w, L, D, H, F, V, tied_embeddings=False)


@pytest.mark.gpu
@pytest.mark.skipif(not has_gpu(), reason="no CUDA device")
@pytest.mark.parametrize("tied", [True, False])
def test_blob_load_matches_set_weight_and_round_trips(tmp_path, tied):
    import torch

    import evk_b200
    from llm_parity import load_weights
    from llm_ref import RefModel

    evk_b200.init(0)
    L, D, H, F, V = 2, 256, 4, 512, 1000
    ref = RefModel(L, D, H, F, V, tied, dtype=1, seed=9)
    w = {("embedding", 0): ref.emb}
    if not tied:
        w[("lm_head", 0)] = ref.lm_head
    for l, ws in enumerate(ref.w):
        for n in ("wqkv", "wo", "w1", "w2"):
            w[(n, l)] = ws[n]
    p = str(tmp_path / "m.evkw")
    evk_b200.write_weight_blob(p, w, L, D, H, F, V, tied_embeddings=tied, dtype=evk_b200.BF16)
    tok = torch.from_numpy(np.random.default_rng(2).integers(0, V, size=(2, 17)).astype(np.int32)).cuda()
    outs = []
    for how in ("set_weight", "load", "save+load"):
        m = evk_b200.Llm(L, D, H, F, V, 2, 32, dtype=evk_b200.BF16, tied_embeddings=tied)
        if how == "set_weight":
            load_weights(m, ref, torch.bfloat16)
            m.save(str(tmp_path / "saved.evkw"))
        elif how == "load":
            m.load(p)
        else:
            m.load(str(tmp_path / "saved.evkw"))
        nxt = torch.zeros(2, dtype=torch.int32, device="cuda")
        lg = torch.empty(2, V, dtype=torch.bfloat16, device="cuda")
        m.prefill(tok, nxt, lg)
        torch.cuda.synchronize()
        outs.append(lg.clone())
        m.close()
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    assert open(p, "rb").read() == open(tmp_path / "saved.evkw", "rb").read()
    # a blob of another configuration is rejected
    m = evk_b200.Llm(L, D, H, F, V + 8, 2, 32, dtype=evk_b200.BF16, tied_embeddings=tied)
    with pytest.raises(evk_b200.EvkcuError):
        m.load(p)
    m.close()
