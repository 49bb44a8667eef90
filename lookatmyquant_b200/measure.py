"""The `measure` sweep's KL probes on B200 (config 4): every linear piece of a model quantized at each trellis option,
one at a time, and the KL of held-out windows to the unquantized model measured after each.

Reference: compiler.py:134-291 (`measure`): held windows and their reference log-probabilities once (:176-187), input
statistics H per group of four layers from a calibration pass that stops after the group (:220-265), then per piece
and option `word(option, W, H, seed, trellis)` (quantize.py:332-347: the column TrellisCode with T = 320 for a
960-wide model, two-sided rotation), the weight swapped in, `kl() − floor` recorded, the weight restored.

Here: H from the tcgen05 statistics kernel (bf16 activations, as the reference's fp32 Xᵀ·X of the bf16 stream), the
word from the column-trellis sweep kernel, the forward through the model's own bf16 layers — from the quantized
piece's layer on, the earlier layers' outputs being kept from the reference pass (Probe) — with the quantized piece
running as a TrellisLinear (the trellis-dequant tensor-core GEMM straight from the word's states and rotations, no
dense weight), and the KL from the fused LM-head/log-softmax/KL kernel (kl.KLReference) on the final hidden states —
no logits are formed. `dense_piece=True` writes the dense word into the model instead, as the reference does. The model is a
random-initialised SmolLM2-360M-architecture Llama (weights N(0, 0.02²), bf16) and the windows are seeded Zipf tokens.
"""

from __future__ import annotations

import json
import time

import torch

from . import codes
from .artifact import TrellisLinear
from .hessian import Statistics
from .kl import KLReference

STAGES = [("self_attn", ["self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"]),
          ("self_attn", ["self_attn.o_proj"]),
          ("mlp", ["mlp.gate_proj", "mlp.up_proj"]),
          ("mlp", ["mlp.down_proj"])]
BLOCK_SEED = {"self_attn": 2, "mlp": 3}  # compiler_arch.block_seed for the Llama blocks


def smollm2_config(layers: int = 32):
    from transformers import LlamaConfig
    cfg = LlamaConfig(hidden_size=960, intermediate_size=2560, num_hidden_layers=layers, num_attention_heads=15,
                      num_key_value_heads=5, vocab_size=49152, rms_norm_eps=1e-5, rope_theta=1e5,
                      tie_word_embeddings=True, max_position_embeddings=8192, initializer_range=0.02)
    cfg._attn_implementation = "sdpa"
    return cfg


def build_model(layers: int = 32, seed: int = 0, device="cuda"):
    """A SmolLM2-360M-architecture model with random N(0, 0.02²) weights, bf16, on the device."""
    from transformers import LlamaForCausalLM
    torch.manual_seed(seed)
    model = LlamaForCausalLM(smollm2_config(layers))
    return model.to(device=device, dtype=torch.bfloat16).eval()


def zipf_tokens(windows: int, T: int, V: int, seed: int, s: float = 1.1) -> torch.Tensor:
    """windows × T token ids, id r − 1 with probability ∝ r^−s (seeded, torch's CPU generator)."""
    w = torch.arange(1, V + 1, dtype=torch.float64).pow(-s)
    g = torch.Generator().manual_seed(seed)
    return torch.multinomial(w, windows * T, replacement=True, generator=g).reshape(windows, T)


class _Stop(Exception):
    pass


@torch.no_grad()
def capture(model, layers, chunks) -> dict:
    """{(layer, first name of the stage): H (fp64)} for the stages of `layers`, from one calibration pass over
    `chunks` that stops after the group's last layer (compiler.py:220-265)."""
    decoder = model.model.layers
    stats, hooks = {}, []
    for i in layers:
        for _, names in STAGES:
            key = (i, names[0])
            mod = decoder[i].get_submodule(names[0])

            def hook(m, a, key=key, d=mod.in_features):
                if key not in stats:
                    stats[key] = Statistics(d, device=a[0].device)
                stats[key].add(a[0].reshape(-1, a[0].shape[-1]))
            hooks.append(mod.register_forward_pre_hook(hook))
    last = max(layers)
    if last + 1 < len(decoder):
        def stop(m, a, k):
            raise _Stop()
        hooks.append(decoder[last + 1].register_forward_pre_hook(stop, with_kwargs=True))
    try:
        for x in chunks:
            try:
                model.model(x, use_cache=False)
            except _Stop:
                pass
    finally:
        for h in hooks:
            h.remove()
    out = {}
    for key, st in stats.items():
        H, _ = st.finalize()
        st.check_status()
        out[key] = H
    return out


class Probe:
    """Held windows, their reference distribution (once) and the KL of the current model to it.

    A probe quantizes one piece of one decoder layer, so the layers before it see exactly the reference model: the
    hidden state entering every layer (and the arguments the model passes to its layers) is kept from the reference
    pass, and `kl(start=i)` runs only layers i, i + 1, … — the same modules on the same inputs, so the hidden states are
    bit-identical to a full forward's, for about half the work on average (the reference re-runs the whole model)."""

    def __init__(self, model, held: torch.Tensor, batch: int = 2, weights: torch.Tensor | None = None,
                 prefix_cache: bool = True):
        self.model, self.held, self.batch = model, held, batch
        self.w = weights
        self.cache = self._capture_prefix() if prefix_cache else None
        self.ref = KLReference(self.hidden(), model.lm_head.weight)

    @torch.no_grad()
    def _capture_prefix(self) -> list:
        """[(layer inputs, layer kwargs)] per batch of windows, from one pass of the unquantized model."""
        dev = self.model.lm_head.weight.device
        cache = []
        for b in range(0, len(self.held), self.batch):
            ins, kw, hooks = [], {}, []

            def pre(m, args, kwargs):
                ins.append(args[0] if args else kwargs["hidden_states"])
                if not kw:
                    kw.update({k: v for k, v in kwargs.items() if k != "hidden_states"})
            for layer in self.model.model.layers:
                hooks.append(layer.register_forward_pre_hook(pre, with_kwargs=True))
            try:
                self.model.model(self.held[b:b + self.batch].to(dev), use_cache=False)
            finally:
                for h in hooks:
                    h.remove()
            cache.append((ins, kw))
        return cache

    @torch.no_grad()
    def hidden(self, start: int | None = None) -> torch.Tensor:
        """The final hidden states of the held windows; with `start`, only layers start, start + 1, … are run, from
        the cached input of layer `start` (the layers before it must be unchanged since the reference pass)."""
        dev = self.model.lm_head.weight.device
        if start is None or self.cache is None:
            hs = [self.model.model(self.held[b:b + self.batch].to(dev), use_cache=False).last_hidden_state
                  for b in range(0, len(self.held), self.batch)]
        else:
            layers = self.model.model.layers
            hs = []
            for ins, kw in self.cache:
                h = ins[start]
                for layer in layers[start:]:
                    h = layer(h, **kw)
                hs.append(self.model.model.norm(h))
        return torch.cat(hs).reshape(-1, hs[0].shape[-1])

    def kl(self, start: int | None = None) -> float:
        return self.ref.kl(self.hidden(start), self.w)


def pieces(layers, n_layers: int) -> list:
    """The linear pieces of `layers` in the reference's measure order (layer, stage, matrix): (layer, block, stage
    index, matrix index, name) each."""
    out = []
    for i in layers:
        for si, (block, names) in enumerate(STAGES):
            for j, name in enumerate(names):
                out.append((i, block, si, j, name))
    return out


def assign_pieces(items: list, n_layers: int, world: int) -> list:
    """Pieces per rank for a sweep split across `world` ranks: each piece (all of its options) goes to one rank, the
    costliest first onto the least loaded rank. A probe of layer i re-runs layers i..n_layers − 1 (the earlier layers'
    outputs are cached), so its cost is taken as n_layers − i + 1. Every rank computes the same assignment from the
    same list; no communication is needed. The reference splits the same item space by layer span, one job each
    (run_batch.py:40-43); pieces balance better than spans because late layers are cheaper to probe."""
    load = [0.0] * world
    owned = [[] for _ in range(world)]
    for k in sorted(range(len(items)), key=lambda k: (-(n_layers - items[k][0] + 1), k)):
        r = min(range(world), key=lambda q: (load[q], q))
        load[r] += n_layers - items[k][0] + 1
        owned[r].append(k)
    return [sorted(o) for o in owned]


def gather_records(res: dict, group, order: list) -> dict:
    """All ranks' records in the single-rank order (`order`: item names in sweep order), with the job's probe count
    and the slowest rank's seconds in probes (what the whole job waits for)."""
    import torch.distributed as dist
    parts = [None] * dist.get_world_size(group)
    dist.all_gather_object(parts, {"records": res["records"], "seconds in probes": res["seconds in probes"],
                                   "probes": res["probes"]}, group=group)
    rank_of = {name: k for k, name in enumerate(order)}
    recs = sorted((r for part in parts for r in part["records"]),
                  key=lambda r: (rank_of[r["item"]], r["option"]))
    slowest = max(part["seconds in probes"] for part in parts)
    probes = sum(part["probes"] for part in parts)
    out = dict(res)
    out.update({"records": recs, "probes": probes, "seconds in probes": slowest,
                "probes per hour": 3600.0 * probes / slowest if slowest else None,
                "seconds in probes per rank": [part["seconds in probes"] for part in parts]})
    return out


def run(layers=range(2), options=("tr2", "tr3", "tr4"), n_layers: int = 32, windows: int = 8, T: int = 2048,
        calib: int = 16, chunk: int = 4, kl_batch: int = 8, seed: int = 0, device="cuda", log=print,
        rank: int = 0, world: int = 1, group=None, dense_piece: bool = False) -> dict:
    """The measure sweep over the linear pieces of `layers`: returns the records and the timing. With world > 1 this
    rank probes only its share of the pieces (assign_pieces) on its own model replica, and with a process group the
    ranks' records are gathered (every rank returns the whole sweep)."""
    dev = torch.device(device)
    t_all = time.time()
    model = build_model(n_layers, seed, dev)
    V = model.config.vocab_size
    held = zipf_tokens(windows, T, V, seed + 1)
    cal = zipf_tokens(calib, T, V, seed + 2)
    chunks = [cal[b:b + chunk].to(dev) for b in range(0, len(cal), chunk)]
    t0 = time.time()
    probe = Probe(model, held, kl_batch)
    torch.cuda.synchronize()
    t_ref = time.time() - t0
    t0 = time.time()
    floor = probe.kl()
    t_kl = time.time() - t0
    T_tr = 256 if model.config.hidden_size % 256 == 0 else 320
    trellis = {}
    recs, t_probe, n_probe = [], 0.0, 0
    layers = list(layers)
    items = pieces(layers, n_layers)
    mine = set(assign_pieces(items, n_layers, world)[rank]) if world > 1 else set(range(len(items)))
    mine_layers = sorted({items[k][0] for k in mine})
    groups = [layers[k:k + 4] for k in range(0, len(layers), 4)]
    for grp in groups:
        if not any(i in mine_layers for i in grp):
            continue
        H = capture(model, grp, chunks)
        for k, (i, block, si, j, name) in enumerate(items):
            if i not in grp or k not in mine:
                continue
            L = model.model.layers[i]
            Hs = H[(i, STAGES[si][1][0])]
            mod = L.get_submodule(name)
            orig = mod.weight.data.clone()
            W = orig.double()
            m, n = W.shape
            Tm = T_tr if m % T_tr == 0 else next(t for t in (320, 256, 128, 64) if m % t == 0)
            seed_ = 1000 * i + 100 * BLOCK_SEED[block] + j
            for o in options:
                kbits = int(o[2:])
                if (kbits, Tm) not in trellis:
                    trellis[(kbits, Tm)] = codes.TrellisCode(12, kbits, T=Tm)
                ts = time.time()
                word = codes.ldlq_words([W], Hs, trellis[(kbits, Tm)], [seed_])[0]
                if dense_piece:
                    mod.weight.data = word.matrix().to(torch.bfloat16)
                    d = probe.kl(start=i) - floor
                    mod.weight.data = orig
                else:
                    parent, leaf = L.get_submodule(name.rsplit(".", 1)[0]), name.rsplit(".", 1)[1]
                    setattr(parent, leaf, TrellisLinear(word))
                    try:
                        d = probe.kl(start=i) - floor
                    finally:
                        setattr(parent, leaf, mod)
                dt = time.time() - ts
                t_probe += dt
                n_probe += 1
                recs.append({"item": f"{i}.{name}", "layer": i, "role": name, "shape": [m, n], "T": Tm,
                             "option": o, "bits": word.rate_bits(), "dkl": d, "seconds": round(dt, 4)})
            log(f"  layer {i} {name}: " + ", ".join(f"{r['option']} {r['dkl']:.3e}" for r in recs[-len(options):]))
    res = {"records": recs, "kl floor": floor, "probes": n_probe, "seconds in probes": t_probe,
           "probes per hour": 3600.0 * n_probe / t_probe if t_probe else None, "seconds per kl": t_kl,
           "seconds for the reference distribution": t_ref, "seconds": time.time() - t_all,
           "held windows": [windows, T], "calibration": [calib, T], "rank": rank, "world": world}
    if group is not None and world > 1:
        res = gather_records(res, group, [f"{i}.{name}" for i, _, _, _, name in items])
    return res


def main():
    """`python -m lookatmyquant_b200.measure [--layers A:B] [--windows 8] [--T 2048]`: the config-4 KL probes over the
    linear pieces of the chosen layers of a random SmolLM2-360M-architecture model; prints one JSON summary. Under
    torch.distributed.run each rank takes its share of the pieces on its own GPU and rank 0 prints the whole sweep."""
    import argparse
    import datetime
    import os
    ap = argparse.ArgumentParser(description=main.__doc__)
    ap.add_argument("--layers", default="0:1")
    ap.add_argument("--model-layers", type=int, default=32)
    ap.add_argument("--windows", type=int, default=8)
    ap.add_argument("--T", type=int, default=2048)
    ap.add_argument("--calib", type=int, default=16)
    ap.add_argument("--options", nargs="+", default=["tr2", "tr3", "tr4"])
    ap.add_argument("--out", default=None)
    a = ap.parse_args()
    lo, hi = (int(x) for x in a.layers.split(":"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank, group = int(os.environ.get("RANK", "0")), None
    device = "cuda"
    if world > 1:
        import torch.distributed as dist
        local = int(os.environ.get("LOCAL_RANK", rank))
        torch.cuda.set_device(local)
        device = f"cuda:{local}"
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
        group = dist.group.WORLD
    res = run(range(lo, hi), a.options, a.model_layers, a.windows, a.T, a.calib, device=device,
              log=print if rank == 0 else (lambda s: None), rank=rank, world=world, group=group)
    if rank == 0:
        summary = {k: v for k, v in res.items() if k != "records"}
        print(json.dumps(summary), flush=True)
        if a.out:
            with open(a.out, "w") as f:
                json.dump(res, f, indent=1)
    if group is not None:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
