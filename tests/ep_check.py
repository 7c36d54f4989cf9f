"""Multi-GPU check of the expert-parallel MoE decoder (run under torchrun, one
process per GPU; invoked by tests/test_gpu_moe_ep.py when the host has >= 2
GPUs). Every rank builds the same small model from host weights; rank r runs
MoeEPModel on its token block with its block of experts, once with the
fixed-capacity exchange (also replayed from its CUDA graph and through the
host entry) and once with the exact host-sized splits; rank 0 also runs the
single-GPU MoeModel over all tokens and compares each rank's rows. A capacity
far below the routed share must raise the exchange-overflow error.

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 tests/ep_check.py <batch>
"""
import os
import sys
from datetime import timedelta
from dataclasses import replace
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def main():
    import torch
    import torch.distributed as dist
    import burn_rocket_b200 as rb
    from burn_rocket_b200.moe import MoeConfig, MoeModel
    from burn_rocket_b200.moe_ep import MoeEPModel, ep_plan
    from oracle import moe_ref

    batch = int(sys.argv[1]) if len(sys.argv) > 1 else 2
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    rb.init(local)
    cfg = replace(MoeConfig(), layers=2, hidden=1024, heads=8, kv_heads=2, head_dim=128, experts=16, top_k=4,
                  inter=256, vocab=512)
    seq = 256
    hw = moe_ref.make_host_weights(cfg, seed=31)
    ids = np.random.default_rng(32).integers(0, cfg.vocab, size=batch * seq, dtype=np.int32)
    pairs = [dist.new_group([2 * i, 2 * i + 1]) for i in range(world // 2)] if world > batch else None
    mine = np.concatenate([ids[s * seq + r0: s * seq + r0 + n] for s, r0, n in ep_plan(world, batch, seq)[rank]])
    outs = {}
    # fixed-capacity exchange (no host reads; captured into a CUDA graph) and the exact host-sized splits
    for mode, factor in (("capacity", 1.25), ("exact", None), ("calibrated", 1.25)):
        model = MoeEPModel(cfg, batch, seq, rank, world, host_weights=hw, pair_groups=pairs, capacity_factor=factor)
        model.ids_in.copy_(torch.from_numpy(mine))
        if mode == "calibrated":
            cap = model.calibrate_capacity()
            print(f"rank {rank}: calibrated capacity {cap} of {model.S} slots", flush=True)
        out = model.forward_device().float().clone()
        rb.check_device_errors()
        if factor is not None:
            model.capture()
            replay = model.run().float().clone()
            torch.cuda.synchronize()
            assert torch.equal(replay, out), "graph replay differs from the eager forward"
            host = model.prefill_host(torch.from_numpy(mine).pin_memory()).float()
            assert torch.equal(host, out.cpu()), "host entry differs"
            model.graph = None
        outs[mode] = out
        del model
        torch.cuda.synchronize()
    # a capacity far below the routed share: the overflow is flagged, not silent
    small = MoeEPModel(cfg, batch, seq, rank, world, host_weights=hw, pair_groups=pairs, capacity_factor=0.05)
    small.ids_in.copy_(torch.from_numpy(mine))
    small.forward_device()
    try:
        rb.check_device_errors()
        overflow_flagged = False
    except rb.OpFailure as e:
        overflow_flagged = "overflow" in str(e)
    del small
    status = torch.zeros(1, device="cuda")
    status[0] = 1.0 if overflow_flagged else 0.0
    gathered = {m: [torch.empty_like(o) for _ in range(world)] for m, o in outs.items()}
    for m, o in outs.items():
        dist.all_gather(gathered[m], o)
    if rank == 0:
        ref = MoeModel(cfg, batch, seq, host_weights=hw)
        ref.ids_in.copy_(torch.from_numpy(ids))
        want = ref.forward_device().float().cpu().numpy()
        plan = ep_plan(world, batch, seq)
        worst = 1.0
        for m in outs:
            for r in range(world):
                rows = np.concatenate([np.arange(s * seq + r0, s * seq + r0 + n) for s, r0, n in plan[r]])
                a, b = gathered[m][r].cpu().numpy().ravel().astype(np.float64), want[rows].ravel().astype(np.float64)
                cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
                worst = min(worst, cos)
                print(f"{m} exchange, rank {r}: cosine vs single-GPU {cos:.7f}", flush=True)
        same = all(torch.equal(gathered[m][r], gathered["exact"][r]) for m in ("capacity", "calibrated")
                   for r in range(world))
        print(f"capacity, calibrated == exact exchange: {same}; overflow flagged: {overflow_flagged}", flush=True)
        status[0] = status[0] * (1.0 if worst >= 0.9999 and same else 0.0)
    dist.all_reduce(status, op=dist.ReduceOp.MIN)
    ok = bool(status.item() == 1.0)
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
