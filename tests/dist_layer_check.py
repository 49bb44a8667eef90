"""Worker of test_gpu_multi.py, launched by torch.distributed.run with one process per GPU: a small two-stage layer
built with its tokens and rows sharded over the ranks (H and D all-reduced after every stage's statistics, the stages'
factorizations on rank pairs — each stage on its own pair with 4 or more ranks — and broadcast), every rank's
states gathered to rank 0 and compared with the same layer built on one GPU."""

import datetime
import os
import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


def main():
    from lookatmyquant_b200.layer import StageSpec, build_layer
    from lookatmyquant_b200.workloads import config3, token_shard
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                         device_id=torch.device("cuda", local))
    rank, world = torch.distributed.get_rank(), torch.distributed.get_world_size()
    dev = torch.device("cuda", local)
    spec = [StageSpec("attn_in", 512, [("self_attn.q_proj", 512), ("self_attn.k_proj", 256)], "self_attn"),
            StageSpec("down_in", 1024, [("mlp.down_proj", 512)], "mlp")]
    tokens = 65536
    lo, hi = token_shard(tokens, rank, world)
    stages, weights, acts, w, bits = config3(tokens, device=dev, lo=lo, hi=hi, stages=spec)
    group = torch.distributed.group.WORLD
    if world >= 2:  # every stage's statistics first, the stages' factorizations on rank pairs
        from lookatmyquant_b200.hessian import Statistics
        from lookatmyquant_b200.layer import build_stages_sharded
        stats = []
        for s in stages:
            x, xr = acts[s.name]
            st = Statistics(s.d, cross=True, device=dev)
            st.add(x, w, xr)
            stats.append(st)
        out = build_stages_sharded(stages, weights, stats, bits, group=group, dequantize=False, n_tok_total=tokens)
    else:
        out = build_layer(stages, weights, acts, w, bits, group=group, dequantize=False, n_tok_total=tokens)
    torch.cuda.synchronize()
    parts = [None] * world
    mine = {s.name: {nm: (out[s.name].row_range[nm], out[s.name].states[nm].cpu()) for nm in out[s.name].states}
            for s in stages}
    torch.distributed.all_gather_object(parts, mine)
    ok = True
    if rank == 0:
        _, w1, a1, ww, b1 = config3(tokens, device=dev, stages=spec)
        ref = build_layer(stages, w1, a1, ww, b1, dequantize=False)
        for s in stages:
            for nm, rows in s.matrices:
                full = torch.full((rows, s.d), -1, dtype=torch.int16)
                for p in parts:
                    if nm in p[s.name]:
                        (a, b), t = p[s.name][nm]
                        full[a:b] = t
                same = float((full == ref[s.name].states[nm].cpu()).double().mean())
                print(f"{s.name} {nm}: {same:.5f} of the states equal the one-GPU build", flush=True)
                ok &= same >= 0.999
    torch.distributed.barrier()
    torch.distributed.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
