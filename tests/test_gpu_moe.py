"""Device parity of the MoE layer pieces and of the config #5 (Qwen3-30B-A3B
style) decoder against the CPU oracle (oracle/moe_ref.py, itself pinned to the
reference's golden MoE decoder in tests/test_oracle_moe.py).

Routing is compared exactly wherever the oracle's top-k margin (the gap
between the k-th and the (k+1)-th probability, src/clef/model.rs:462-489)
exceeds what f32 rounding can move; weights within 1e-6. Expert outputs and
hidden states (the 2-layer forward with the oracle following the device's
routing): cosine >= 0.9999 and max |err| <= 1e-2 * max |ref|.
"""
import math
from dataclasses import replace

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def max_rel(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.abs(got - want).max() / (np.abs(want).max() + 1e-30))


def cosine(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-300))


def test_route_matches_oracle(rb):
    import torch
    import burn_rocket_b200._lib as L
    from oracle import moe_ref
    lib = L.load()
    rng = np.random.default_rng(5)
    T, E, K = 777, 128, 8
    logits = rng.standard_normal((T, E)).astype(np.float32)
    logits[0, :] = 1.0            # all tied: ids 0..7, weights 1/8
    logits[1, [3, 9, 40]] = 5.0   # tie inside the selection
    ld = torch.from_numpy(logits).cuda()
    ids = torch.empty(T, K, dtype=torch.int32, device="cuda")
    wts = torch.empty(T, K, dtype=torch.float32, device="cuda")
    assert lib.rb_moe_route(ld.data_ptr(), T, E, K, 1, ids.data_ptr(), wts.data_ptr(), None) == 0, L.last_error()
    got_i, got_w = ids.cpu().numpy(), wts.cpu().numpy()
    want_i, want_w, margin = moe_ref.route(logits, K)
    assert got_i[0].tolist() == list(range(8)) and np.allclose(got_w[0], 0.125, atol=1e-7)
    assert got_i[1, :3].tolist() == [3, 9, 40]
    stable = margin > 1e-6
    assert stable.mean() > 0.95
    assert np.array_equal(got_i[stable], want_i[stable])
    assert np.abs(got_w[stable] - want_w[stable]).max() < 1e-6
    # unnormalised weights
    assert lib.rb_moe_route(ld.data_ptr(), T, E, K, 0, ids.data_ptr(), wts.data_ptr(), None) == 0
    _, raw_w, _ = moe_ref.route(logits, K, norm=False)
    assert np.abs(wts.cpu().numpy()[stable] - raw_w[stable]).max() < 1e-6
    assert lib.rb_moe_route(ld.data_ptr(), T, 300, K, 1, ids.data_ptr(), wts.data_ptr(), None) != 0  # E > 256


def test_dispatch_grouped_gemm_combine_matches_oracle(rb, orc):
    """route -> dispatch -> grouped gate|up -> SiLU·mul -> grouped down -> combine."""
    import torch
    import burn_rocket_b200 as rbm
    import burn_rocket_b200._lib as L
    from oracle import moe_ref
    lib = L.load()
    rng = np.random.default_rng(6)
    T, E, K, H, I = 300, 16, 4, 1024, 256
    x16 = rng.standard_normal((T, H)).astype(np.float16)
    x0 = rng.standard_normal((T, H)).astype(np.float32)
    ids_np, w_np, _ = moe_ref.route(rng.standard_normal((T, E)), K)
    experts = [((rng.standard_normal((I, H)) * 0.02).astype(np.float32),
                (rng.standard_normal((I, H)) * 0.02).astype(np.float32),
                (rng.standard_normal((H, I)) * 0.02).astype(np.float32)) for _ in range(E)]
    gu_id = rbm._pack_parts_q8_0([m for g, u, _ in experts for m in (g, u)])
    dn_id = rbm._pack_parts_q8_0([d for _, _, d in experts])
    rows = int(lib.rb_moe_max_rows(T, K, E))
    ws = torch.empty(int(lib.rb_moe_workspace_bytes(T, K, E)) // 4 + 1, dtype=torch.int32, device="cuda")
    xd = torch.from_numpy(x16).cuda()
    ids = torch.from_numpy(ids_np.astype(np.int32)).cuda()
    wts = torch.from_numpy(w_np.astype(np.float32)).cuda()
    xp = torch.empty(rows, H, dtype=torch.float16, device="cuda")
    gup = torch.empty(rows, 2 * I, dtype=torch.float16, device="cuda")
    act = torch.empty(rows, I, dtype=torch.float16, device="cuda")
    yp = torch.empty(rows, H, dtype=torch.float16, device="cuda")
    xres = torch.from_numpy(x0).cuda()
    assert lib.rb_moe_dispatch(ids.data_ptr(), T, K, E, xd.data_ptr(), H, ws.data_ptr(), xp.data_ptr(), None) == 0
    assert lib.rb_matmul_grouped(gu_id.id, E, xp.data_ptr(), rows, ws.data_ptr(), T, K, gup.data_ptr(),
                                 L.DTYPE_F16, None) == 0, L.last_error()
    assert lib.rb_silu_mul_halves(gup.data_ptr(), rows, I, act.data_ptr(), None) == 0
    assert lib.rb_matmul_grouped(dn_id.id, E, act.data_ptr(), rows, ws.data_ptr(), T, K, yp.data_ptr(),
                                 L.DTYPE_F16, None) == 0, L.last_error()
    assert lib.rb_moe_combine(xres.data_ptr(), yp.data_ptr(), H, ids.data_ptr(), wts.data_ptr(), ws.data_ptr(),
                              T, K, E, None) == 0
    got = xres.cpu().numpy().astype(np.float64) - x0
    rb.check_device_errors()
    deq = lambda w: orc.q8_0_dequant(*orc.q8_0_quantize(w)).astype(np.float64)
    want = moe_ref.experts_combine(np.zeros((T, H)), x16.astype(np.float64), ids_np, w_np,
                                   [(deq(g), deq(u), deq(d)) for g, u, d in experts])
    assert cosine(got, want) >= 0.9999, cosine(got, want)
    assert max_rel(got, want) <= 1e-2, max_rel(got, want)


SMALL = dict(layers=2, hidden=1024, heads=8, kv_heads=2, head_dim=128, experts=16, top_k=4, inter=256, vocab=512)


def test_moe_forward_matches_oracle(rb):
    import torch
    from burn_rocket_b200.moe import MoeConfig, MoeModel
    from oracle import moe_ref
    cfg = replace(MoeConfig(), **SMALL)
    batch, seq = 2, 128
    hw = moe_ref.make_host_weights(cfg, seed=21)
    model = MoeModel(cfg, batch, seq, host_weights=hw)
    ids = np.random.default_rng(22).integers(0, cfg.vocab, size=batch * seq, dtype=np.int32)
    model.ids_in.copy_(torch.from_numpy(ids))
    got = model.forward_device(record_routing=True).float().cpu().numpy()
    rb.check_device_errors()
    want, routing = moe_ref.forward(hw, cfg, ids, batch, seq)
    # routing of the first layer: exact where the oracle's selection is stable
    # (device logits differ from the f64 oracle by ~1e-4 relative, so a
    # selection whose top-k margin exceeds 1e-3 cannot flip)
    stable_all = np.ones(batch * seq, bool)
    for li, (rid, rw, margin) in enumerate(routing):
        dev_ids = model.routing[li][0].cpu().numpy()
        stable = margin > 1e-3
        assert stable.mean() > 0.7, (li, stable.mean())
        # the selected set (its order can swap between near-equal selected experts;
        # the combine sums in ascending expert id either way)
        assert np.array_equal(np.sort(dev_ids[stable], 1), np.sort(rid[stable], 1)), li
        stable_all &= stable
    # the whole forward, with the oracle chain following the device's routing
    # (a near-tie flip changes which experts a token uses, which no tolerance
    # on the outputs can absorb; the selection itself is checked above)
    forced, _ = moe_ref.forward(hw, cfg, ids, batch, seq,
                                force_routing=[r[0].cpu().numpy() for r in model.routing])
    for b in range(batch):
        rows = slice(b * seq, (b + 1) * seq)
        assert cosine(got[rows], forced[rows]) >= 0.9999, (b, cosine(got[rows], forced[rows]))
    assert max_rel(got, forced) <= 1e-2, max_rel(got, forced)


def test_moe_graph_replay_equals_eager(rb):
    import torch
    from burn_rocket_b200.moe import MoeConfig, MoeModel
    cfg = replace(MoeConfig(), **SMALL)
    model = MoeModel(cfg, 2, 128, seed=4)
    model.ids_in.copy_(torch.randint(0, cfg.vocab, (256,), dtype=torch.int32))
    eager = model.forward_device().clone()
    model.capture()
    replay = model.run().clone()
    torch.cuda.synchronize()
    assert torch.equal(eager, replay)
    rb.check_device_errors()
