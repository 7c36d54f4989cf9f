"""Host-side logic of the expert-parallel exchange (burn_rocket_b200/moe_ep.py)
on CPU with world_size-2 gloo process groups: token-block ownership
(`ep_plan`), the send-buffer bookkeeping (`build_send_np`, the restatement of
rb_ep_build_send), the uneven all-to-all (`exchange`) both ways, and the
expert-id-ordered combine — checked against the same computation in one
process."""
import os
import socket

import numpy as np
import pytest

from burn_rocket_b200.moe_ep import build_send_fixed_np, build_send_np, ep_plan, exchange

E, K, H = 8, 3, 16


def expert_fn(rows, experts):
    """A stand-in expert: row * (e + 1) + e (each expert distinguishable)."""
    return rows * (experts[:, None] + 1.0) + experts[:, None]


def combine(x, ids, w, outs_by_slot):
    """x[t] += sum over slots in ascending expert id of w * out (src/clef/engine.rs:317-340)."""
    y = x.copy()
    for t in range(ids.shape[0]):
        for j in np.argsort(ids[t], kind="stable"):
            y[t] += w[t, j] * outs_by_slot[t * K + j]
    return y


def rank_inputs(rank, tokens):
    rng = np.random.default_rng(100 + rank)
    ids = np.array([rng.choice(E, K, replace=False) for _ in range(tokens)], dtype=np.int64).reshape(tokens, K)
    w = rng.random((tokens, K)).astype(np.float32)
    x = rng.standard_normal((tokens, H)).astype(np.float32)
    return ids, w, x


def worker(rank, world, port, tokens, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ids, w, x = rank_inputs(rank, tokens[rank])
        counts, meta, slot_pos = build_send_np(ids, E, world)
        send_rows = np.empty((ids.size, H), np.float32)
        send_rows[slot_pos] = np.repeat(x, K, axis=0)  # slot s carries token s // K
        rc = torch.empty(world, dtype=torch.int64)
        exchange(rc, torch.from_numpy(counts), [1] * world, [1] * world)
        recv_splits = rc.tolist()
        R = sum(recv_splits)
        recv_rows = torch.empty(R, H)
        recv_meta = torch.empty(R, dtype=torch.int64)
        exchange(recv_rows, torch.from_numpy(send_rows), recv_splits, counts.tolist())
        exchange(recv_meta, torch.from_numpy(meta.astype(np.int64)), recv_splits, counts.tolist())
        global_e = recv_meta.numpy() + rank * (E // world)
        y_recv = torch.from_numpy(expert_fn(recv_rows.numpy(), global_e).astype(np.float32))
        y_back = torch.empty(ids.size, H)
        exchange(y_back, y_recv, counts.tolist(), recv_splits)
        outs_by_slot = y_back.numpy()[slot_pos]
        q.put((rank, combine(x, ids, w, outs_by_slot)))
    finally:
        dist.destroy_process_group()


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("tokens", [(37, 29), (5, 0)])
def test_ep_exchange_matches_single_process(tokens):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, 2, port, tokens, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=60) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        ids, w, x = rank_inputs(r, tokens[r])
        flat = ids.reshape(-1)
        want = combine(x, ids, w, expert_fn(np.repeat(x, K, axis=0), flat))
        np.testing.assert_allclose(results[r], want, rtol=1e-6, atol=1e-6)


def test_ep_plan():
    assert ep_plan(2, 4, 2048) == [[(0, 0, 2048), (1, 0, 2048)], [(2, 0, 2048), (3, 0, 2048)]]
    assert ep_plan(8, 4, 2048)[5] == [(2, 1024, 1024)]
    with pytest.raises(ValueError):
        ep_plan(3, 4, 2048)


def test_build_send_groups_slots_by_destination():
    ids = np.array([[0, 5], [7, 2], [4, 1]])
    counts, meta, pos = build_send_np(ids, 8, 2)
    assert counts.tolist() == [3, 3]
    dest = ids.reshape(-1) // 4
    assert (dest[np.argsort(pos)] == np.sort(dest, kind="stable")).all()
    assert (meta[pos] == ids.reshape(-1) % 4).all()


def worker_fixed(rank, world, port, tokens, capacity, q):
    """The fixed-capacity exchange: equal all-to-all splits of `capacity` rows,
    padding rows (meta -1) skipped by the experts, slots past the capacity
    dropped and flagged."""
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ids, w, x = rank_inputs(rank, tokens[rank])
        _, meta, slot_pos, overflow = build_send_fixed_np(ids, E, world, capacity)
        send_rows = np.zeros((world * capacity, H), np.float32)
        sent = slot_pos >= 0
        send_rows[slot_pos[sent]] = np.repeat(x, K, axis=0)[sent]
        recv_rows = torch.empty(world * capacity, H)
        recv_meta = torch.empty(world * capacity, dtype=torch.int64)
        exchange(recv_rows, torch.from_numpy(send_rows), None, None)
        exchange(recv_meta, torch.from_numpy(meta), None, None)
        rm = recv_meta.numpy()
        y_recv = np.zeros((world * capacity, H), np.float32)
        real = rm >= 0
        y_recv[real] = expert_fn(recv_rows.numpy()[real], rm[real] + rank * (E // world))
        y_back = torch.empty(world * capacity, H)
        exchange(y_back, torch.from_numpy(y_recv), None, None)
        outs_by_slot = np.zeros((ids.size, H), np.float32)
        outs_by_slot[sent] = y_back.numpy()[slot_pos[sent]]
        q.put((rank, combine(x, ids, w, outs_by_slot), overflow))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("tokens,capacity", [((37, 29), 64), ((5, 0), 8), ((37, 29), 4)])
def test_ep_fixed_capacity_exchange(tokens, capacity):
    """Equal splits of a fixed capacity reproduce the single-process result
    whenever no destination overflows; an overflow is reported."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker_fixed, args=(r, 2, port, tokens, capacity, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict((r, (y, of)) for r, y, of in (q.get(timeout=120) for _ in procs))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(2):
        ids, w, x = rank_inputs(r, tokens[r])
        y, overflow = got[r]
        counts = np.bincount(ids.reshape(-1) // (E // 2), minlength=2)
        assert overflow == bool((counts > capacity).any())
        if not overflow:
            want = combine(x, ids, w, expert_fn(np.repeat(x, K, axis=0), ids.reshape(-1).astype(np.float32)))
            np.testing.assert_allclose(y, want, rtol=1e-6, atol=1e-6)
