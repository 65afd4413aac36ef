"""GPU: one process drives two GPUs (the reference's engine does, docs/multi-gpu-layer.md).

Kernel attributes such as the dynamic shared-memory limit belong to a device, so a
context on a second device must set them there too. Contexts on devices 0 and 1
score config-2-shaped pages (fp16 K, 24 / 4 heads, head_dim 256, pages of 256
tokens) and pick the top-k, each checked against the FP64 oracle and the picker.
Skipped with fewer than two GPUs.
"""
import numpy as np
import pytest

from tests import util as U

pytestmark = pytest.mark.gpu


def test_contexts_on_two_devices():
    import torch

    import kvmem_b200 as K
    from oracle import oracle as O
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    L, Hq, Hkv, D, T, page, budget = 2, 24, 4, 256, 8192, 256, 8
    P = T // page
    scale = float(np.float32(1) / np.sqrt(np.float32(D)))
    for dev_i in (1, 0, 1):  # device 1 first: nothing may rely on device 0 having been set up
        rng = np.random.default_rng(dev_i)
        kb = U.make_k(rng, U.F16, L, T, Hkv, D)
        qb = U.make_q(rng, U.F32, L, 1, Hq, D)
        dev = torch.device("cuda", dev_i)
        with torch.cuda.device(dev):
            k_d = torch.from_numpy(kb.reshape(-1).copy()).to(dev)
            q_d = torch.from_numpy(qb.reshape(-1).copy()).to(dev).view(torch.float32).view(L, 1, Hq, D)
            ctx = K.RecallContext(dev_i)
            desc = K.RecallContext.make_desc(layers=L, q_heads=Hq, kv_heads=Hkv, head_dim=D, tokens=T,
                                             page_tokens=page)
            kc = K.RecallContext.make_kcache(k_d, U.F16, kv_heads=Hkv, head_dim=D, capacity_tokens=T)
            stream = torch.cuda.current_stream(dev)
            _, mean = ctx.score_pages(desc, K.RecallContext.make_query(q_d, 1), kc, want_rows=False, stream=stream)
            ids, n = ctx.select_topk(mean.view(L, P), [0, P - 1], budget, stream=stream)
            torch.cuda.synchronize(dev)
            ctx.check_status(f"device {dev_i}", stream=stream)
            got = mean.cpu().numpy().reshape(L, P)
            ids_h, n_h = ids.cpu().numpy(), n.cpu().numpy()
            ctx.close()
        exp = O.page_mass(qb, U.F32, kb, U.F16, layers=L, rows=1, heads=Hq, kv_heads=Hkv, dim=D, tokens=T,
                          page_tokens=page, scale=scale)[:, 0, 0]
        ok, worst, nbad = U.close(got, exp, 1e-3, 1e-6)
        assert ok, f"device {dev_i}: {nbad} masses off, worst {worst:.3g}"
        for l in range(L):
            rc, want = O.pick_scored(P, list(range(P)), got[l].astype(np.float64), [0, P - 1], budget)
            assert rc == 0 and ids_h[l, : n_h[l]].tolist() == want.tolist()
