"""Expert-parallel form of the MoE decoder (BASELINE config #5 on 2/4/8 GPUs).

One process per GPU. The 128 experts are split into `world` consecutive
blocks (rank r owns experts [r*E/world, (r+1)*E/world)); the dense part
(attention, router) runs on the rank that owns the token:

  * world <= batch: rank r owns whole sequences (data parallel);
  * world == 2 * batch: rank r owns half a sequence. The second half's
    attention needs the first half's K/V, so each pair of ranks all-gathers
    its k|v columns and the second half runs a causal block mask with query
    offset seq/2 (`attention_causal_block`).

Per layer the routed slots travel to their experts' ranks and back with NCCL
all-to-alls of f16 token rows (plus one of the local expert ids):

    route -> rb_ep_build_send_capacity -> all_to_all(rows, meta)
      -> local grouped expert GEMMs -> all_to_all(outputs back)
      -> rb_moe_combine_rows (ascending expert id per token, as
         src/clef/engine.rs:317-340)

The exchange has a fixed capacity per destination (capacity_factor x the even
share of the rank's routed slots, default 1.25, or calibrate_capacity() from
an exact forward over the actual inputs): every split is `capacity` rows,
padding rows carry expert id -1 and are skipped, so no count is read on the
host and the whole forward is captured into one CUDA graph. A routing so
skewed that a destination receives more than its capacity sets the
exchange-overflow bit of the device error word (rb_check_device_errors); a
caller then reruns the step with capacity_factor=None (the exact form, which
reads the per-destination counts on the host every layer and sizes each
all-to-all to them) or recalibrates. The buffers are sized for the worst case
(every slot to one destination), so the capacity can change freely.

The reference runs every expert on one board (experts streamed from NVMe,
src/clef/engine.rs:7-19); expert parallelism is new here.
"""
from __future__ import annotations

import ctypes as C
import math

import numpy as np

from . import _lib
from . import _check, _dev_ptr, WeightId, matmul, pack_gated_q8_0
from ._lib import DTYPE_F16, MASK_CAUSAL, MASK_CAUSAL_BLOCK
from .moe import MoeConfig
from .qwen3 import rope_tables


def ep_plan(world: int, batch: int, seq: int):
    """Per rank: (sequence index, first row within the sequence, rows) of the
    token block it owns, as a list of blocks."""
    if world <= batch:
        if batch % world:
            raise ValueError(f"world {world} must divide the batch of {batch} sequences")
        per = batch // world
        return [[(r * per + i, 0, seq) for i in range(per)] for r in range(world)]
    if world == 2 * batch and seq % 2 == 0:
        return [[(r // 2, (r % 2) * (seq // 2), seq // 2)] for r in range(world)]
    raise ValueError(f"world {world} must divide the batch ({batch}) or be twice it")


def exchange(out, inp, out_splits, in_splits, group=None):
    """all_to_all_single along dim 0 (NCCL for CUDA tensors, gloo for CPU
    tensors): uneven splits, or equal ones when the splits are None."""
    import torch.distributed as dist
    if out_splits is None:
        dist.all_to_all_single(out, inp, group=group)
    else:
        dist.all_to_all_single(out, inp, list(map(int, out_splits)), list(map(int, in_splits)), group=group)
    return out


# ---------------------------------------------------------------- host restatement (tests)
def build_send_np(ids: np.ndarray, experts: int, ranks: int):
    """numpy restatement of rb_ep_build_send with a stable (slot-order) layout:
    counts [ranks], meta [slots] (expert id local to the destination),
    slot_pos [slots] (send position of every slot)."""
    per = experts // ranks
    flat = ids.reshape(-1)
    dest = flat // per
    counts = np.bincount(dest, minlength=ranks).astype(np.int64)
    order = np.argsort(dest, kind="stable")
    slot_pos = np.empty_like(order)
    slot_pos[order] = np.arange(order.size)
    meta = (flat - dest * per)[order]
    return counts, meta, slot_pos


def build_send_fixed_np(ids: np.ndarray, experts: int, ranks: int, capacity: int):
    """numpy restatement of rb_ep_build_send_capacity with a stable (slot-order)
    layout: counts [ranks], meta [ranks*capacity] (local expert id, -1 where
    unused), slot_pos [slots] (send position, -1 for a slot past its
    destination's capacity) and whether any destination overflowed."""
    per = experts // ranks
    flat = ids.reshape(-1)
    dest = flat // per
    counts = np.bincount(dest, minlength=ranks).astype(np.int64)
    meta = np.full(ranks * capacity, -1, np.int64)
    slot_pos = np.full(flat.size, -1, np.int64)
    fill = np.zeros(ranks, np.int64)
    for s in range(flat.size):
        q = dest[s]
        if fill[q] < capacity:
            pos = q * capacity + fill[q]
            meta[pos] = flat[s] - q * per
            slot_pos[s] = pos
        fill[q] += 1
    return counts, meta, slot_pos, bool((counts > capacity).any())


class MoeEPModel:
    """Expert-parallel MoE decoder: this rank's token blocks, all dense
    weights, and its own block of experts (Q8_0)."""

    def __init__(self, cfg: MoeConfig, batch: int, seq: int, rank: int, world: int, seed: int = 0,
                 host_weights: dict | None = None, group=None, pair_groups=None,
                 capacity_factor: float | None = 1.25):
        import torch
        self.cfg, self.batch, self.seq, self.rank, self.world = cfg, batch, seq, rank, world
        self.group = group
        self.blocks = ep_plan(world, batch, seq)[rank]
        self.split = world > batch  # half sequences
        self.pair_group = pair_groups[rank // 2] if self.split else None
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        self.T = sum(b[2] for b in self.blocks)
        T = self.T
        lib = _lib.load()
        E, I, h, d, nh, nkv, k = cfg.experts, cfg.inter, cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads, cfg.top_k
        if E % world:
            raise ValueError("experts must divide over the ranks")
        self.epr = E // world
        e0 = rank * self.epr
        g_dense = torch.Generator(device=dev).manual_seed(seed)
        g_exp = torch.Generator(device=dev).manual_seed(seed * 1000 + 7 + rank)

        def randn(gen, *shape):
            return torch.randn(*shape, generator=gen, device=dev, dtype=torch.float32).mul_(0.02)

        def pack_dev(parts):
            parts = [p.float().contiguous() for p in parts]
            ptrs = (C.c_void_p * len(parts))(*[p.data_ptr() for p in parts])
            ns = (C.c_int64 * len(parts))(*[p.shape[0] for p in parts])
            wid = lib.rb_pack_f32_q8_0_device(ptrs, ns, len(parts), parts[0].shape[1])
            _check(wid, "rocket_pack", 0, parts[0].shape[1], sum(p.shape[0] for p in parts))
            return WeightId(int(wid))

        self.gated = I % 64 == 0  # fused gate|up + silu_mul epilogue
        epr = self.epr

        def pack_gu(gate, up):
            return pack_gated_q8_0(gate, up) if self.gated else pack_dev(
                [m for e in range(epr) for m in (gate[e * I:(e + 1) * I], up[e * I:(e + 1) * I])])

        self.layers = []
        for li in range(cfg.layers):
            if host_weights is not None:
                W = host_weights["layers"][li]
                t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)
                layer = {"qkv": pack_dev([t(W["wq"]), t(W["wk"]), t(W["wv"])]), "o": pack_dev([t(W["wo"])]),
                         "router": pack_dev([t(W["router"])]),
                         "gu": pack_gu(torch.cat([t(gate) for gate, _, _ in W["experts"][e0:e0 + self.epr]]),
                                       torch.cat([t(up) for _, up, _ in W["experts"][e0:e0 + self.epr]])),
                         "down": pack_dev([t(dn) for _, _, dn in W["experts"][e0:e0 + self.epr]])}
                layer.update({kk: t(W[kk]) for kk in ("in_norm", "post_norm", "q_norm", "k_norm")})
            else:
                layer = {"qkv": pack_dev([randn(g_dense, nh * d, h), randn(g_dense, nkv * d, h),
                                          randn(g_dense, nkv * d, h)]),
                         "o": pack_dev([randn(g_dense, h, nh * d)]), "router": pack_dev([randn(g_dense, E, h)])}
                gate, up = randn(g_exp, self.epr * I, h), randn(g_exp, self.epr * I, h)
                layer["gu"] = pack_gu(gate, up)
                del gate, up
                big = randn(g_exp, self.epr * h, I)
                layer["down"] = pack_dev([big])
                del big
                ones = lambda n: torch.ones(n, device=dev)
                layer.update({"in_norm": ones(h), "post_norm": ones(h), "q_norm": ones(d), "k_norm": ones(d)})
            self.layers.append(layer)
        if host_weights is not None:
            self.final_norm = torch.from_numpy(host_weights["final_norm"]).to(dev).float()
            self.embed = torch.from_numpy(host_weights["embed"]).to(dev).half().contiguous()
        else:
            self.final_norm = torch.ones(h, device=dev)
            self.embed = (torch.randn(cfg.vocab, h, generator=g_dense, device=dev) * 0.02).half().contiguous()
        cos, sin = rope_tables(seq, d, cfg.theta)
        self.cos = torch.from_numpy(cos).to(dev)
        self.sin = torch.from_numpy(sin).to(dev)
        torch.cuda.synchronize()
        f16 = torch.float16
        S = T * k                      # slots sent by this rank
        self.S = S
        # exchange buffers for the worst case: every slot of every rank to one
        # destination (world * S rows), whatever the capacity
        R = S_buf = world * S
        self.capacity = None if capacity_factor is None else min(
            S, max(8, int(math.ceil(capacity_factor * S / world / 8.0)) * 8))
        self.R_cap = R
        self.max_dest = 0  # largest per-destination row count seen by an exact forward
        self.ids_in = torch.zeros(T, dtype=torch.int32, device=dev)
        self.x = torch.empty(T, h, dtype=torch.float32, device=dev)
        self.h = torch.empty(T, h, dtype=f16, device=dev)
        self.qkv = torch.empty(T, (nh + 2 * nkv) * d, dtype=f16, device=dev)
        self.kv_full = torch.empty(2 * T, 2 * nkv * d, dtype=f16, device=dev) if self.split else None
        self.attn = torch.empty(T, nh * d, dtype=f16, device=dev)
        self.o = torch.empty(T, h, dtype=f16, device=dev)
        self.logits = torch.empty(T, E, dtype=torch.float32, device=dev)
        self.ids = torch.empty(T, k, dtype=torch.int32, device=dev)
        self.wts = torch.empty(T, k, dtype=torch.float32, device=dev)
        self.dest_counts = torch.empty(world, dtype=torch.int32, device=dev)
        self.recv_counts = torch.empty(world, dtype=torch.int32, device=dev)
        self.dest_cursor = torch.empty(world, dtype=torch.int32, device=dev)
        self.send_meta = torch.empty(S_buf, dtype=torch.int32, device=dev)
        self.slot_pos = torch.empty(S, dtype=torch.int32, device=dev)
        self.send_rows = torch.empty(S_buf, h, dtype=f16, device=dev)
        self.recv_meta = torch.empty(R, dtype=torch.int32, device=dev)
        self.recv_rows = torch.empty(R, h, dtype=f16, device=dev)
        self.y_recv = torch.empty(R, h, dtype=f16, device=dev)
        self.y_back = torch.empty(S_buf, h, dtype=f16, device=dev)
        self.max_rows = int(lib.rb_moe_max_rows(R, 1, self.epr))
        self.ws = torch.empty(int(lib.rb_moe_workspace_bytes(R, 1, self.epr)) // 4 + 1, dtype=torch.int32,
                              device=dev)
        self.xp = torch.empty(self.max_rows, h, dtype=f16, device=dev)
        self.gup = None if self.gated else torch.empty(self.max_rows, 2 * I, dtype=f16, device=dev)
        self.actp = torch.empty(self.max_rows, I, dtype=f16, device=dev)
        self.yp = torch.empty(self.max_rows, h, dtype=f16, device=dev)
        self.out = torch.empty(T, h, dtype=f16, device=dev)
        self.exchanged_rows = 0
        self.graph = None

    def _attention(self, L, lib, qkv_p, ld, st):
        cfg, d, nh, nkv = self.cfg, self.cfg.head_dim, self.cfg.heads, self.cfg.kv_heads
        scale = 1.0 / math.sqrt(d)
        if not self.split:
            b = len(self.blocks)
            _check(lib.rb_attention_batched(qkv_p, ld, qkv_p + nh * d * 2, ld, qkv_p + (nh + nkv) * d * 2, ld,
                                            _dev_ptr(self.attn), nh * d, DTYPE_F16, b, self.seq, self.seq,
                                            nh, nkv, d, scale, 0.0, MASK_CAUSAL, -1, 0, 0, st),
                   "rocket_flash_attn", self.seq, self.seq, d)
            return
        import torch.distributed as dist
        half = self.seq // 2
        # all-gather the pair's k|v column blocks: rows [0, half) then [half, seq)
        kv_mine = self.qkv[:, nh * d:].contiguous()
        dist.all_gather_into_tensor(self.kv_full, kv_mine, group=self.pair_group)
        kvp = _dev_ptr(self.kv_full)
        ldkv = 2 * nkv * d
        q_start = self.blocks[0][1]
        n_kv = q_start + half
        _check(lib.rb_attention_batched(qkv_p, ld, kvp, ldkv, kvp + nkv * d * 2, ldkv, _dev_ptr(self.attn), nh * d,
                                        DTYPE_F16, 1, half, n_kv, nh, nkv, d, scale, 0.0, MASK_CAUSAL_BLOCK, -1,
                                        q_start, 0, st),
               "rocket_flash_attn", half, n_kv, d)

    def _experts(self, L, lib, R, st):
        """Grouped expert GEMMs over R received rows (recv_meta, recv_rows) into
        y_recv in receive order."""
        cfg = self.cfg
        h, I = cfg.hidden, cfg.inter
        rows = int(lib.rb_moe_max_rows(R, 1, self.epr))
        ws = _dev_ptr(self.ws)
        _check(lib.rb_moe_dispatch(_dev_ptr(self.recv_meta), R, 1, self.epr, _dev_ptr(self.recv_rows), h,
                                   ws, _dev_ptr(self.xp), st), "moe_dispatch")
        if self.gated:  # silu(gate x) * (up x) straight from the grouped GEMM
            _check(lib.rb_matmul_grouped(L["gu"].id, self.epr, _dev_ptr(self.xp), rows, ws, R, 1,
                                         _dev_ptr(self.actp), DTYPE_F16, st), "matmul_grouped")
        else:
            _check(lib.rb_matmul_grouped(L["gu"].id, self.epr, _dev_ptr(self.xp), rows, ws, R, 1,
                                         _dev_ptr(self.gup), DTYPE_F16, st), "matmul_grouped")
            _check(lib.rb_silu_mul_halves(_dev_ptr(self.gup), rows, I, _dev_ptr(self.actp), st), "silu_mul")
        _check(lib.rb_matmul_grouped(L["down"].id, self.epr, _dev_ptr(self.actp), rows, ws, R, 1,
                                     _dev_ptr(self.yp), DTYPE_F16, st), "matmul_grouped")
        # back to receive order: y_recv[i] = yp[row of received slot i] (padding slots: none)
        off = int(lib.rb_moe_slot_rows_offset(R, 1, self.epr))
        _check(lib.rb_gather_rows(_dev_ptr(self.yp), ws + 4 * off, R, h, _dev_ptr(self.y_recv), st),
               "gather_rows")

    def forward_device(self, exact: bool = False):
        """One forward over self.ids_in (this rank's tokens) into self.out, on
        the current CUDA stream; exact=True (or no capacity set) sizes every
        all-to-all to the per-destination counts, read on the host."""
        from . import _stream_ptr
        cap = None if exact else self.capacity
        cfg, lib, T = self.cfg, _lib.load(), self.T
        h, d, nh, nkv, E, k = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads, cfg.experts, cfg.top_k
        W = self.world
        st = _stream_ptr(None)
        ld = (nh + 2 * nkv) * d
        qkv_p, xp = _dev_ptr(self.qkv), _dev_ptr(self.x)
        # rope positions of this rank's first row (tables offset by the row within the sequence)
        pos0 = self.blocks[0][1]
        cos_p = _dev_ptr(self.cos) + pos0 * (d // 2) * 4
        sin_p = _dev_ptr(self.sin) + pos0 * (d // 2) * 4
        rope_seq = self.blocks[0][2]
        _check(lib.rb_embed_gather(_dev_ptr(self.ids_in), T, _dev_ptr(self.embed), cfg.vocab, h, xp, st),
               "embed_gather")
        self.exchanged_rows = 0
        for L in self.layers:
            _check(lib.rb_add_rms_norm(xp, None, _dev_ptr(L["in_norm"]), cfg.eps, _dev_ptr(self.h), T, h, st),
                   "add_rms_norm")
            matmul(self.h, L["qkv"], out=self.qkv)
            _check(lib.rb_qk_norm_rope(qkv_p, ld, T, nh, nkv, d, _dev_ptr(L["q_norm"]), _dev_ptr(L["k_norm"]),
                                       cfg.eps, cos_p, sin_p, rope_seq, st), "qk_norm_rope")
            self._attention(L, lib, qkv_p, ld, st)
            matmul(self.attn, L["o"], out=self.o)
            _check(lib.rb_add_rms_norm(xp, _dev_ptr(self.o), _dev_ptr(L["post_norm"]), cfg.eps, _dev_ptr(self.h),
                                       T, h, st), "add_rms_norm")
            matmul(self.h, L["router"], out=self.logits)
            _check(lib.rb_moe_route(_dev_ptr(self.logits), T, E, k, 1, _dev_ptr(self.ids), _dev_ptr(self.wts), st),
                   "moe_route")
            if cap is not None:
                # fixed-capacity exchange: equal splits, nothing read on the host
                _check(lib.rb_ep_build_send_capacity(_dev_ptr(self.ids), T, k, E, W, cap,
                                                     _dev_ptr(self.h), h, _dev_ptr(self.dest_counts),
                                                     _dev_ptr(self.dest_cursor), _dev_ptr(self.send_meta),
                                                     _dev_ptr(self.slot_pos), _dev_ptr(self.send_rows), st),
                       "ep_build_send_capacity")
                n = W * cap
                exchange(self.recv_rows[:n], self.send_rows[:n], None, None, self.group)
                exchange(self.recv_meta[:n], self.send_meta[:n], None, None, self.group)
                self._experts(L, lib, n, st)
                exchange(self.y_back[:n], self.y_recv[:n], None, None, self.group)
            else:
                # exact splits: the per-destination counts are read on the host
                _check(lib.rb_ep_build_send(_dev_ptr(self.ids), T, k, E, W, _dev_ptr(self.h), h,
                                            _dev_ptr(self.dest_counts), _dev_ptr(self.dest_cursor),
                                            _dev_ptr(self.send_meta), _dev_ptr(self.slot_pos),
                                            _dev_ptr(self.send_rows), st), "ep_build_send")
                exchange(self.recv_counts, self.dest_counts, [1] * W, [1] * W, self.group)
                send_splits = self.dest_counts.cpu().tolist()
                recv_splits = self.recv_counts.cpu().tolist()
                R = int(sum(recv_splits))
                self.exchanged_rows += int(sum(send_splits))
                self.max_dest = max(self.max_dest, max(send_splits))
                S = self.S
                exchange(self.recv_rows[:R], self.send_rows[:S], recv_splits, send_splits, self.group)
                exchange(self.recv_meta[:R], self.send_meta[:S], recv_splits, send_splits, self.group)
                if R > 0:
                    self._experts(L, lib, R, st)
                exchange(self.y_back[:S], self.y_recv[:R], send_splits, recv_splits, self.group)
            _check(lib.rb_moe_combine_rows(xp, _dev_ptr(self.y_back), h, _dev_ptr(self.ids), _dev_ptr(self.wts),
                                           _dev_ptr(self.slot_pos), T, k, st), "moe_combine")
        _check(lib.rb_add_rms_norm(xp, None, _dev_ptr(self.final_norm), cfg.eps, _dev_ptr(self.out), T, h, st),
               "add_rms_norm")
        return self.out

    def calibrate_capacity(self, margin: float = 1.05) -> int:
        """Set the exchange capacity from an exact forward over the current
        inputs: the largest per-destination row count over every layer and
        rank, times `margin`, rounded up to 8 (at most every slot). All ranks
        call it together and agree on the result."""
        import torch
        import torch.distributed as dist
        self.max_dest = 0
        self.forward_device(exact=True)
        t = torch.tensor([self.max_dest], dtype=torch.int64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
        self.capacity = min(self.S, max(8, int(math.ceil(int(t.item()) * margin / 8.0)) * 8))
        self.graph = None
        return self.capacity

    def capture(self):
        """Capture forward_device (fixed-capacity exchange) into a CUDA graph,
        NCCL all-to-alls included, after one eager warm-up."""
        import torch
        if self.capacity is None:
            raise RuntimeError("only the fixed-capacity exchange is graph-capturable")
        self.forward_device()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, capture_error_mode="thread_local"):
            self.forward_device()
        self.graph = g
        return g

    def run(self):
        if self.graph is not None:
            self.graph.replay()
        else:
            self.forward_device()
        return self.out

    def prefill_host(self, ids_host, out_host=None):
        """End-to-end call: this rank's host token ids in, its final-normed f16 hidden states out."""
        import torch
        self.ids_in.copy_(ids_host, non_blocking=True)
        self.run()
        if out_host is None:
            out_host = torch.empty(self.T, self.cfg.hidden, dtype=torch.float16, pin_memory=True)
        out_host.copy_(self.out, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return out_host
