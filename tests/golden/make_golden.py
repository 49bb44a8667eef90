"""Generate the golden vectors that pin the oracle, by running the reference itself (CPU) on seeded inputs.

Run from the repository root, in a container where the reference checkout is available:

    python tests/golden/make_golden.py --reference <path to the lookatmyquant checkout>

The reference reads a model config at import (opgraph/model.py:37-47) and writes fitted trellis tables next to its
sources (opgraph/codes.py:42); both are redirected to a temporary directory, the reference's files are only read. The
outputs are small `.npz` fixtures in this directory, plus the reference's four fitted L=12 trellis tables
(cache/codes/trellis_L12_k{1,2,3,4}_T256_s0_ema.pt, fp64 data) re-encoded as raw little-endian fp64 under
lookatmyquant_b200/tables/, where the package and the tests read them on machines without the reference.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import shutil
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
TABLES = REPO / "lookatmyquant_b200" / "tables"

SMOLLM2 = {"hidden_size": 960, "num_attention_heads": 15, "num_key_value_heads": 5, "intermediate_size": 2560,
           "num_hidden_layers": 32, "rms_norm_eps": 1e-5, "rope_theta": 100000.0, "vocab_size": 49152,
           "tie_word_embeddings": True, "model_type": "llama"}


def setup_reference(ref: Path):
    home = Path(tempfile.mkdtemp(prefix="lamq_ref_home_"))
    snap = home / ".cache/huggingface/hub/models--HuggingFaceTB--SmolLM2-360M/snapshots/x"
    snap.mkdir(parents=True)
    (snap / "config.json").write_text(json.dumps(SMOLLM2))
    os.environ["HOME"] = str(home)
    os.environ["OPGRAPH_DEVICE"] = "cpu"
    os.environ["PYTHONDONTWRITEBYTECODE"] = "1"
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(ref))
    import opgraph.codes as C
    cache = home / "codes"
    shutil.copytree(ref / "cache" / "codes", cache)
    C.CACHE = cache
    return C


def calib_H(n, tokens, seed, dead=()):
    """Config-1-style statistics: Gaussian tokens, per-channel std lognormal(0, 1), 4 outlier channels ×20;
    H = XᵀX / tokens, rounded to fp32 values so the fixture stores it exactly."""
    import torch
    g = torch.Generator().manual_seed(seed)
    std = torch.exp(torch.randn(n, generator=g, dtype=torch.float64))
    out = torch.randperm(n, generator=g)[:4]
    std[out] *= 20
    X = torch.randn(tokens, n, generator=g, dtype=torch.float64) * std
    for d in dead:
        X[:, d] = 0
    H = (X.T @ X / tokens).float().double()
    return H


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--only", choices=["artifact", "fit", "neartie", "ldlq_gpu", "statistics", "kl", "best_word",
                                       "embedding", "importance", "finetune", "dropin", "small_l"],
                    help="write only this fixture (the others stay as committed)")
    ap.add_argument("--case", type=Path, help="for --only neartie: an .npz with X (1 x T), values (4096) and k")
    args = ap.parse_args()
    C = setup_reference(args.reference.resolve())
    import torch
    import quantize as Q
    import compiler_artifact as CA
    from opgraph.frame import Environment

    if args.only == "artifact":
        write_artifact_fixture(C, Q, CA, torch)
        return
    if args.only == "fit":
        write_fit_fixture(C, torch)
        return
    if args.only == "neartie":
        write_neartie_fixture(C, torch, args.case)
        return
    if args.only == "ldlq_gpu":
        write_ldlq_gpu_fixture(torch, Environment)
        return
    if args.only == "statistics":
        write_statistics_fixture(torch, args.reference.resolve())
        return
    if args.only == "kl":
        write_kl_fixture(torch, Q)
        return
    if args.only == "best_word":
        write_best_word_fixture(C, Q, torch, args.reference.resolve())
        return
    if args.only == "embedding":
        write_embedding_fixture(Q, torch)
        return
    if args.only == "importance":
        write_importance_fixture(Q, torch, args.reference.resolve())
        return
    if args.only == "finetune":
        write_finetune_fixture(C, torch)
        return
    if args.only == "dropin":
        write_dropin_fixture(C, Q, torch)
        return
    if args.only == "small_l":
        write_small_l_fixture(C, torch)
        return
    # the reference's fitted L=12 tables, as raw fp64
    TABLES.mkdir(parents=True, exist_ok=True)
    digests = {}
    for k in (1, 2, 3, 4):
        v = C.trellis_values(12, k, 256).double().numpy()
        path = TABLES / f"trellis_L12_k{k}_T256_s0_ema.f64"
        path.write_bytes(v.astype("<f8").tobytes())
        digests[path.name] = hashlib.sha256(path.read_bytes()).hexdigest()
    # the sums cover every table in the folder (the T = 320 ones are fitted on the GPU by `python -m
    # lookatmyquant_b200.codes fit`, which reproduces these T = 256 tables bit for bit)
    for path in TABLES.glob("trellis_*.f64"):
        digests.setdefault(path.name, hashlib.sha256(path.read_bytes()).hexdigest())
    (TABLES / "SHA256SUMS").write_text("".join(f"{h}  {n}\n" for n, h in sorted(digests.items())))

    # 1. Viterbi (codes.py:151-181): windows with a start state, free-start runs, small tables
    vit = {}
    g = torch.Generator().manual_seed(11)
    for k in (1, 2, 3, 4):
        v = C.trellis_values(12, k, 256)
        X = torch.randn(48, 24, generator=g, dtype=torch.float64).float().double()
        start = torch.randint(0, 4096, (48,), generator=g)
        vit[f"k{k}_X"] = X.numpy()
        vit[f"k{k}_start"] = start.numpy()
        vit[f"k{k}_states_start"] = C.viterbi(X, v, 12, k, start=start).numpy()
        X2 = torch.randn(8, 256, generator=g, dtype=torch.float64).float().double()
        vit[f"k{k}_Xfree"] = X2.numpy()
        vit[f"k{k}_states_free"] = C.viterbi(X2, v, 12, k).numpy()
        X3 = torch.randn(16, 7, generator=g, dtype=torch.float64).float().double()  # short windows (T < 8)
        vit[f"k{k}_Xshort"] = X3.numpy()
        vit[f"k{k}_states_short"] = C.viterbi(X3, v, 12, k, start=torch.zeros(16, dtype=torch.long)).numpy()
    v8 = torch.randn(256, generator=g, dtype=torch.float64).float().double()
    X8 = torch.randn(32, 40, generator=g, dtype=torch.float64).float().double()
    vit["L8_values"], vit["L8_X"], vit["L8_states"] = v8.numpy(), X8.numpy(), C.viterbi(X8, v8, 8, 2).numpy()
    v4 = torch.randn(16, generator=g, dtype=torch.float64).float().double()
    X4 = torch.randn(5, 7, generator=g, dtype=torch.float64).float().double()
    vit["L4_values"], vit["L4_X"], vit["L4_states"] = v4.numpy(), X4.numpy(), C.viterbi(X4, v4, 4, 1).numpy()
    np.savez_compressed(HERE / "viterbi.npz", **vit)

    # 2. Hadamard rotations (codes.py:97-132)
    rot = {}
    for n, seed in ((64, 5), (200, 7), (256, 301), (320, 9), (960, 301), (2560, 1301), (4096, 2201), (9728, 3301)):
        A, B = C.hadamard_factors(n)
        R = C.rht(n, seed)
        rot[f"n{n}_seed"] = np.array(seed)
        rot[f"n{n}_shapes"] = np.array([A.shape[0], B.shape[0]])
        rot[f"n{n}_rows"] = R[:2].numpy()
        vec = torch.randn(n, generator=torch.Generator().manual_seed(n), dtype=torch.float64)
        rot[f"n{n}_Rv"] = (R @ vec).numpy()
        del R
    np.savez_compressed(HERE / "rotation.npz", **rot)

    # 3. Environment (frame.py:515-522), with a dead input
    H = calib_H(128, 1024, 3, dead=(5,))
    env = Environment(H)
    np.savez_compressed(HERE / "environment.npz", H=H.float().numpy(), U=env.U.numpy(), dead=env.dead.numpy())

    # 4. Row-trellis LDLQ words (codes.py:413-462 with RowTrellisCode, the lm2 path), pack_trellis
    ldlq = {}
    cases = [("a", 64, 256, 2, 300, 301), ("b", 48, 320, 3, 1200, 1201), ("c", 32, 200, 1, 7, 8), ("d", 32, 256, 4, 5, 6)]
    for name, m, n, k, seed, in_seed in cases:
        gW = torch.Generator().manual_seed(1000 + m + n + k)
        W = (0.02 * torch.randn(m, n, generator=gW, dtype=torch.float64)).float().double()
        H = calib_H(n, 2048, 17 + k)
        code = C.RowTrellisCode(12, k, T=256, width=16, look=8)
        net = C.ldlq_words([W], H, code, [seed], in_seed=in_seed, out_rot=False)[0]
        Wq = net.matrix(dtype=torch.float64)
        E = Wq - W
        states = Q.trellis_states(net.cores["W"].data, code.values)
        ldlq[f"{name}_W"] = W.float().numpy()
        ldlq[f"{name}_H"] = H.float().numpy()
        ldlq[f"{name}_meta"] = np.array([m, n, k, seed, in_seed])
        ldlq[f"{name}_states"] = states.numpy()
        ldlq[f"{name}_S"] = net.cores["W.S"].data.numpy()
        ldlq[f"{name}_Wq"] = Wq.float().numpy()
        ldlq[f"{name}_proxy"] = np.array(float((E @ H * E).sum()))
        ldlq[f"{name}_packed"] = CA.pack_trellis(states.numpy().astype(np.int64), k)
    # no rotation, with a dead input (syntax.py:100-101)
    m, n, k = 32, 128, 2
    W = (0.02 * torch.randn(m, n, generator=torch.Generator().manual_seed(77), dtype=torch.float64)).float().double()
    H = calib_H(n, 1024, 23, dead=(3, 40))
    code = C.RowTrellisCode(12, k, T=256, width=16, look=8)
    net = C.ldlq_words([W], H, code, [0], incoherent=False)[0]
    ldlq["e_W"], ldlq["e_H"], ldlq["e_meta"] = W.float().numpy(), H.float().numpy(), np.array([m, n, k, 0, -1])
    ldlq["e_states"] = Q.trellis_states(net.cores["W"].data, code.values).numpy()
    ldlq["e_S"] = net.cores["W.S"].data.numpy()
    ldlq["e_Wq"] = net.matrix(dtype=torch.float64).float().numpy()
    np.savez_compressed(HERE / "ldlq_row.npz", **ldlq)

    # 5. Row groups (quantize.py:530-565) through the reference's own `word` (quantize.py:332-347)
    m, n = 256, 256
    W = (0.02 * torch.randn(m, n, generator=torch.Generator().manual_seed(5), dtype=torch.float64)).float().double()
    H = calib_H(n, 2048, 31)
    perm = torch.randperm(m, generator=torch.Generator().manual_seed(6))
    groups = [{"rows": perm[:64], "bits": 2}, {"rows": perm[64:128], "bits": 1}, {"rows": perm[128:192], "bits": 3},
              {"rows": perm[192:], "bits": 2}]
    trellis = {b: C.RowTrellisCode(12, b, T=256, width=16, look=8) for b in (1, 2, 3, 4)}
    in_seed = 3301

    def round_group(rows, bits):
        return Q.word(f"tr{bits}x", W[rows], H, 3300, trellis, in_seed, False)

    Wq, rate, entry = Q.quantize_row_groups(W, groups, round_group, in_seed, True)
    grp = {"W": W.float().numpy(), "H": H.float().numpy(), "perm": perm.numpy(), "bits": np.array([2, 1, 3, 2]),
           "in_seed": np.array(in_seed), "Wq": Wq.float().numpy(), "states": entry["states"].numpy(),
           "scales": entry["scales"].numpy(), "rate": np.array(rate)}
    np.savez_compressed(HERE / "row_groups.npz", **grp)

    # 6. Column trellis (TrellisCode, codes.py:363-383; the `measure` path, two-sided rotation)
    m, n, k = 256, 64, 2
    W = (0.02 * torch.randn(m, n, generator=torch.Generator().manual_seed(9), dtype=torch.float64)).float().double()
    H = calib_H(n, 1024, 41)
    code = C.TrellisCode(12, k, T=256)
    net = C.ldlq_words([W], H, code, [40])[0]
    col = {"W": W.float().numpy(), "H": H.float().numpy(), "meta": np.array([m, n, k, 40, 256]),
           "Wq": net.matrix(dtype=torch.float64).float().numpy(), "settled": net.cores["W"].data.numpy().reshape(m, n),
           "S": net.cores["W.S"].data.numpy()}
    np.savez_compressed(HERE / "column_trellis.npz", **col)
    write_artifact_fixture(C, Q, CA, torch)
    write_fit_fixture(C, torch)
    write_statistics_fixture(torch, args.reference.resolve())
    write_kl_fixture(torch, Q)
    write_best_word_fixture(C, Q, torch, args.reference.resolve())
    write_embedding_fixture(Q, torch)
    write_importance_fixture(Q, torch, args.reference.resolve())
    write_finetune_fixture(C, torch)
    write_dropin_fixture(C, Q, torch)
    write_small_l_fixture(C, torch)
    print("golden vectors written to", HERE)


def write_ldlq_gpu_fixture(torch, Environment):
    """10. Scalar-level LDLQ (opgraph/ldlq_gpu.py, the rounding of nested.py:117-119) and the generic sweep
    (opgraph/syntax.py:86-124) with a Python projection, by the reference on seeded inputs: ldlq_factor of a
    lognormally scaled H (and of one needing more damping), ldlq_round to 8 and 16 levels with blocks of 128 and 48
    over 192 inputs, and syntax.sweep with a nearest-level projection at width 1 and 4 with a dead input."""
    from opgraph import syntax
    from opgraph.ldlq_gpu import ldlq_factor, ldlq_round
    g = torch.Generator().manual_seed(11)
    n, rows = 192, 70
    A = torch.randn(2 * n, n, generator=g, dtype=torch.float64) * torch.exp(torch.randn(n, generator=g,
                                                                                       dtype=torch.float64))
    H = A.T @ A / (2 * n)
    X = torch.randn(rows, n, generator=g, dtype=torch.float64)
    out = {"H": H.numpy(), "X": X.numpy()}
    U = ldlq_factor(H)
    out["U"] = U.numpy()
    for nl, block in ((8, 128), (16, 48)):
        lv = torch.sort(torch.randn(nl, generator=g, dtype=torch.float64) * 1.2).values
        out[f"levels{nl}"] = lv.numpy()
        out[f"Q{nl}_b{block}"] = ldlq_round(X, U, lv, block=block).numpy()
    # an H that needs more than the first damping: one eigenvalue pushed far below zero
    ev, V = torch.linalg.eigh(H[:64, :64])
    ev[0] = -0.05 * ev.mean()
    Hbad = (V * ev) @ V.T
    out["Hbad"], out["Ubad"] = Hbad.numpy(), ldlq_factor(Hbad).numpy()
    # the generic sweep with a nearest-level projection, a dead input
    Hd = H.clone()  # input 5 is dead: its row and column of H are zero
    Hd[5, :] = 0
    Hd[:, 5] = 0
    env = Environment(Hd)
    lv = torch.as_tensor(out["levels8"])
    mids = (lv[1:] + lv[:-1]) / 2

    def nearest(j, cols, T):
        return lv[torch.bucketize(cols.contiguous(), mids)]
    out["sweep_w1"] = syntax.sweep(X, env, nearest, width=1, lazy=64).numpy()
    out["sweep_w4"] = syntax.sweep(X, env, nearest, width=4, lazy=64).numpy()
    np.savez_compressed(HERE / "ldlq_gpu.npz", **out)


def _reference_code(path: Path, outer: str, pick):
    """Compiled statements of the reference, taken from its source as written: the function definitions and
    statements inside `outer` (at any depth) for which pick(ast node, source text) holds, in source order. They run
    below on seeded tensors, so the golden vectors come from the reference's own expressions, not a restatement."""
    import ast
    tree = ast.parse(path.read_text())
    fn = next(n for n in ast.walk(tree) if isinstance(n, ast.FunctionDef) and n.name == outer)
    found = []
    for node in ast.walk(fn):
        if isinstance(node, (ast.stmt,)) and node is not fn and pick(node, ast.unparse(node)):
            found.append(node)
    found.sort(key=lambda n: n.lineno)
    return [(n.lineno, ast.unparse(n), compile(ast.Module(body=[n], type_ignores=[]), str(path), "exec"))
            for n in found]


def write_statistics_fixture(torch, ref: Path):
    """11. Input statistics by the reference's own code on seeded bf16 activations (statgen.py):
    - frame.covariance (opgraph/frame.py:498-505): Σ x xᵀ over 8192-token fp32 chunks, summed in fp64;
    - quantize_stage's weighted accumulation, run statement by statement from quantize.py as written
      (quantize.py:1389-1391 `wq`, :1457 D +=, :1466 H +=, :1467 n_tok +=, :1470 H = (H / n_tok)...), then its QEP
      target (:1482 M = cross_target(H, (D / n_tok).cpu().double() − H) with cross_target of :1330-1335 at α = 0.5 and
      the default λ) and W·M (:1503).
    Stored: the outputs (fp64) and a digest of the inputs."""
    import types
    sys.path.insert(0, str(HERE))
    import statgen
    import quantize as Q
    import opgraph.codes as C
    from opgraph.frame import covariance
    src = ref / "quantize.py"
    defs = {name: _reference_code(src, "main", lambda n, t, name=name: isinstance(n, ast_def()) and n.name == name)
            for name in ("wq", "cross_target")}
    acc = _reference_code(src, "quantize_stage", lambda n, t: t in (
        "D += grab['r'].T @ wq(c, grab['q'], tkey)", "H += grab['q'].T @ wq(c, grab['q'], tkey)",
        "n_tok += len(grab['q'])"))
    fin = _reference_code(src, "quantize_stage", lambda n, t: t == "H = (H / n_tok).cpu().double()")
    qep = _reference_code(src, "quantize_stage", lambda n, t: t == "M = cross_target(H, (D / n_tok).cpu().double() - H)")
    tgt = _reference_code(src, "quantize_stage", lambda n, t: t.startswith("target = W @ M if parse(p)[2]"))
    assert len(acc) == 3 and len(fin) == 1 and len(qep) == 1 and len(tgt) == 1, (acc, fin, qep, tgt)
    out = {}
    for name, tokens, nchunks, d, weighted in statgen.STAT_CASES:
        xq, xr, w, W = statgen.stat_inputs(name)
        out[f"{name}_digest"] = np.array(statgen.digest(xq + (xr or []) + (w or [])))
        if not weighted:
            out[f"{name}_cov"] = covariance(torch.cat(xq)).numpy()
            out[f"{name}_ntok"] = np.array(tokens * nchunks)
            continue
        ns = {"torch": torch, "guided": None, "token_w": tuple(w), "DEV": "cpu", "C": C,
              "args": types.SimpleNamespace(cross_alpha=statgen.QEP_ALPHA, lam=Q.LAM),
              "parse": lambda p: (None, None, True), "p": "tr2x"}
        for code in (defs["wq"][0][2], defs["cross_target"][0][2]):
            exec(code, ns)
        ns.update(H=torch.zeros(d, d), D=torch.zeros(d, d), n_tok=0, tkey=None)
        for c in range(nchunks):
            ns["c"], ns["grab"] = c, {"q": xq[c].float(), "r": xr[c].float()}
            for _, _, code in acc:
                exec(code, ns)
        Dacc = ns["D"].clone()
        exec(fin[0][2], ns)
        exec(qep[0][2], ns)
        ns["W"] = W
        exec(tgt[0][2], ns)
        out[f"{name}_H"] = ns["H"].numpy()
        out[f"{name}_D"] = ((Dacc / ns["n_tok"]).cpu().double() - ns["H"]).numpy()
        if name == "qep":
            out[f"{name}_M"] = ns["M"].numpy()
        out[f"{name}_target"] = ns["target"].numpy()
        out[f"{name}_ntok"] = np.array(ns["n_tok"])
    out["alpha"], out["lam"] = np.array(statgen.QEP_ALPHA), np.array(Q.LAM)
    out["statements"] = np.array([f"quantize.py:{ln}: {t.splitlines()[0]}" for group in
                                  (defs["wq"], defs["cross_target"], acc, fin, qep, tgt) for ln, t, _ in group])
    np.savez_compressed(HERE / "statistics.npz", **out)


def write_best_word_fixture(C, Q, torch, ref: Path):
    """13. best_word (quantize.py:1316-1328), run from the reference's source as written (a closure inside main, with
    --seeds 3): the row-trellis word of the seed whose (E @ H * E).sum() is least, for a 48 x 128 target. Stored: each
    candidate's error (the reference's own expression, evaluated on each candidate word) and the chosen word's
    states and matrix."""
    import types
    code = _reference_code(ref / "quantize.py", "main",
                           lambda n, t: isinstance(n, ast_def()) and n.name == "best_word")[0][2]
    m, n, k, seed, nseeds = 48, 128, 2, 500, 3
    W = (0.02 * torch.randn(m, n, generator=torch.Generator().manual_seed(501), dtype=torch.float64)).float().double()
    H = calib_H(n, 2048, 502)
    trellis = {b: C.RowTrellisCode(12, b, T=256, width=16, look=8) for b in (1, 2, 3, 4)}
    ns = {"torch": torch, "args": types.SimpleNamespace(seeds=nseeds), "trellis_for": lambda rows: trellis,
          "word": Q.word, "parse": Q.parse}
    exec(code, ns)
    best = ns["best_word"](f"tr{k}", W, H, seed)
    errs, mats = [], []
    for t in range(nseeds):  # the candidates, as best_word forms them, to record each one's error
        net = Q.word(f"tr{k}", W, H, seed + 7919 * t, trellis)
        E = net.matrix(dtype=torch.float64) - W
        errs.append(float((E @ H * E).sum()))
        mats.append(net.matrix(dtype=torch.float64))
    chosen = [t for t in range(nseeds) if torch.equal(mats[t], best.matrix(dtype=torch.float64))]
    np.savez_compressed(HERE / "best_word.npz", W=W.float().numpy(), H=H.float().numpy(),
                        meta=np.array([m, n, k, seed, nseeds]), errs=np.array(errs), chosen=np.array(chosen[0]),
                        states=Q.trellis_states(best.cores["W"].data, trellis[k].values).numpy())


def write_embedding_fixture(Q, torch):
    """14. Embedding buckets (quantize.py:350-465) by the reference's own embed_word: a column trellis over runs of
    256 rows after a hidden-dimension rotation, with and without H (a lookup table pads 300 rows to 512), a centred
    bucket, the prng bucket; embedding_buckets and frequency_order."""
    out = {}
    cases = [("a", 512, 64, "tr2", 7001, True, False), ("b", 300, 64, "tr3", 7002, False, False),
             ("c", 256, 64, "tr2", 7003, True, True), ("d", 100, 64, "prng", 7004, False, False),
             ("e", 256, 128, "tr4", 7005, True, False)]
    for name, rows, n, prog, seed, with_h, center in cases:
        W = (0.02 * torch.randn(rows, n, generator=torch.Generator().manual_seed(seed), dtype=torch.float64)).float().double()
        H = calib_H(n, 1024, seed + 1) if with_h else None
        net = Q.embed_word(W, H, prog, seed, center=center)
        out[f"{name}_W"] = W.float().numpy()
        if H is not None:
            out[f"{name}_H"] = H.float().numpy()
        out[f"{name}_meta"] = np.array([rows, n, seed, int(with_h), int(center)])
        out[f"{name}_prog"] = np.array(prog)
        out[f"{name}_Q"] = net.matrix(dtype=torch.float64).numpy()
        out[f"{name}_bits"] = np.array(float(net.rate_bits()))
    out["buckets_49152"] = np.array(Q.embedding_buckets(49152))
    out["buckets_1000"] = np.array(Q.embedding_buckets(1000))
    ids = torch.randint(0, 500, (4000,), generator=torch.Generator().manual_seed(9))
    out["freq_ids"] = ids.numpy()
    out["freq_order"] = Q.frequency_order(ids, 600).numpy()
    np.savez_compressed(HERE / "embedding.npz", **out)


def write_importance_fixture(Q, torch, ref: Path):
    """15. Row importance (row_importance.py:57-93) and GuidedQuant token weights (quantize.py:853-894) on a tiny
    random-init fp32 Llama (statgen.tiny_llama; its weights are stored): the importances E[g²]·E[y²] accumulated by
    the reference's own hooks (the `keep` closure of row_importance.main, run from its source) over three windows
    whose sampled tokens are recorded, and the reference's guided_weights itself (its draws recorded too)."""
    import torch.nn.functional as F
    sys.path.insert(0, str(HERE))
    import statgen
    model = statgen.tiny_llama()
    for p in model.parameters():
        p.requires_grad_(False)
    layers = model.model.layers
    mods = {f"{l}.{n}": m for l, L in enumerate(layers) for n, m in L.named_modules() if isinstance(m, torch.nn.Linear)}
    g = torch.Generator().manual_seed(42)
    windows = torch.randint(0, 1000, (3, 32), generator=g)
    weight = (torch.rand(3, 32, generator=g) < 0.5).float()  # the positions that count (the reference's digits)
    keep_code = _reference_code(ref / "row_importance.py", "main",
                                lambda n, t: isinstance(n, ast_def()) and n.name == "keep")[0][2]
    gg = {k: torch.zeros(m.out_features, dtype=torch.float64) for k, m in mods.items()}
    yy = {k: torch.zeros(m.out_features, dtype=torch.float64) for k, m in mods.items()}
    ns = {"gg": gg, "yy": yy, "torch": torch}
    exec(keep_code, ns)
    hooks = [m.register_forward_hook(ns["keep"](k)) for k, m in mods.items()]
    gen = torch.Generator().manual_seed(0)
    sampled = []
    for i in range(len(windows)):  # the window loop of row_importance.py:66-80 (digit mask given as `weight`)
        x = windows[i:i + 1]
        emb = model.get_input_embeddings()(x).detach().requires_grad_(True)
        lg = model(inputs_embeds=emb, use_cache=False).logits.float()
        with torch.no_grad():
            y = torch.multinomial(F.softmax(lg[0], -1), 1, generator=gen)[:, 0]
        sampled.append(y)
        lp = F.log_softmax(lg[0], -1).gather(1, y[:, None])[:, 0]
        (lp * weight[i]).sum().backward()
    for h in hooks:
        h.remove()
    out = {"windows": windows.numpy(), "weight": weight.numpy(), "sampled": torch.stack(sampled).numpy()}
    for k in mods:
        out[f"imp_{k}"] = (gg[k] * yy[k]).clamp_min(1e-30).numpy()
    out["mods"] = np.array(list(mods))
    # GuidedQuant: the reference's function; its draws recorded by wrapping torch.multinomial for the call
    chunks = [windows[:2], windows[2:]]
    base = [torch.ones(2, 32), torch.ones(1, 32) * 2.0]
    stages_of = {i: [{"kind": "linear", "names": [n for n, m in L.named_modules() if isinstance(m, torch.nn.Linear)]}]
                 for i, L in enumerate(layers)}
    draws, real = [], torch.multinomial

    def recording(*a, **k):
        r = real(*a, **k)
        draws.append(r.clone())
        return r
    torch.multinomial = recording
    try:
        gw = Q.guided_weights(model, chunks, stages_of, layers, base, 0.1)
    finally:
        torch.multinomial = real
    out["guided_draws"] = torch.stack([d[:, 0] for d in draws]).numpy()
    for k, v in gw.items():
        out[f"guided_{k}"] = torch.cat(v).numpy()
    out["state"] = np.array(list(model.state_dict().keys()))
    for i, (k, v) in enumerate(model.state_dict().items()):
        out[f"p{i}"] = v.to(torch.bfloat16).view(torch.int16).numpy()
    np.savez_compressed(HERE / "importance.npz", **out)


def write_finetune_fixture(C, torch):
    """16. The fine-tuning's trellis parts by the reference itself (finetune_lib.py): `rounded` — a 96 x 256 W in three
    row groups (k = 1, 2, 3, the shipped tables) under the rotated statistics of a calibration H, scales refitted — and
    TrellisCoded.nearest / repick of a stored entry after a seeded summed gradient."""
    import finetune_lib as FL
    from opgraph.frame import Environment
    m, n, in_seed = 96, 256, 5101
    W = (0.02 * torch.randn(m, n, generator=torch.Generator().manual_seed(5100), dtype=torch.float64)).float()
    H = calib_H(n, 2048, 5102)
    R = FL.FastRHT(n, in_seed)
    env = Environment(FL.rotated_moment(H, R))
    perm = torch.randperm(m, generator=torch.Generator().manual_seed(5103))
    groups = [(perm[32 * i:32 * (i + 1)], k, FL.RowPath(C.trellis_values(12, k, 256), k)) for i, k in enumerate((1, 2, 3))]
    scale0 = R.back(W).double().pow(2).mean(1).sqrt().float()
    scale = scale0.clone()
    P, states = FL.rounded(W, R, groups, scale, env)
    out = {"W": W.numpy(), "H": H.float().numpy(), "in_seed": np.array(in_seed), "perm": perm.numpy(),
           "scale0": scale0.numpy(), "P": P.numpy(), "states": states.numpy(), "scale": scale.numpy()}
    # rows given: the second group's first 10 rows and the third's last 6, in that order
    rows = torch.cat([perm[32:42], perm[90:96]])
    scale2 = scale0.clone()
    P2, states2 = FL.rounded(W, R, groups, scale2, env, rows=rows)
    out.update({"rows2": rows.numpy(), "P2": P2.numpy(), "states2": states2.numpy(), "scale2": scale2.numpy()})
    # a stored entry (the k = 2 group as a matrix of its own) and one proximal re-pick step
    g2 = groups[1][0]
    entry = {"states": states[g2].long().clone(), "scales": scale[g2].clone(),
             "table": C.trellis_values(12, 2, 256).float(), "in_seed": in_seed}
    entry_states = entry["states"].numpy().copy()  # TrellisCoded keeps (and repick overwrites) the tensor itself
    tc = FL.TrellisCoded(entry, {}, move=True)
    acc = 0.8 * torch.randn(tc.states.shape, generator=torch.Generator().manual_seed(5104))
    tc.acc.copy_(acc)
    out.update({"entry_states": entry_states, "entry_scales": entry["scales"].numpy().copy(),
                "acc": acc.numpy(), "eta": np.array(0.7), "nearest": tc.nearest(0.7, 1 << 28).numpy().copy()})
    changed = tc.repick(0.7, 1 << 28)
    out["changed"] = np.array(changed)
    out["k"] = np.array(tc.k)
    np.savez_compressed(HERE / "finetune.npz", **out)


def write_dropin_fixture(C, Q, torch):
    """17. The reference's own call sites, recorded: quantize_row_groups (quantize.py:530-565) over a 192 x 256 matrix
    in three width groups, each through the reference's `word` (quantize.py:332-347), with every call it makes to
    opgraph.codes.ldlq_words and opgraph.codes.viterbi recorded (arguments and results). A test replays each call into
    this package's function of the same name: equal results at every call site mean the patched reference would
    follow the same path, call for call."""
    m, n = 192, 256
    W = (0.02 * torch.randn(m, n, generator=torch.Generator().manual_seed(6001), dtype=torch.float64)).float().double()
    H = calib_H(n, 2048, 6002)
    perm = torch.randperm(m, generator=torch.Generator().manual_seed(6003))
    groups = [{"rows": perm[:64], "bits": 2}, {"rows": perm[64:128], "bits": 3}, {"rows": perm[128:], "bits": 1}]
    trellis = {b: C.RowTrellisCode(12, b, T=256, width=16, look=8) for b in (1, 2, 3, 4)}
    in_seed = 6101
    vit_calls, words_calls = [], []
    real_v, real_w = C.viterbi, C.ldlq_words

    def spy_viterbi(X, values, L, k, chunk=None, start=None):
        out = real_v(X, values, L, k, chunk=chunk, start=start)
        vit_calls.append((X.clone(), k, None if start is None else start.clone(), out.clone()))
        return out

    def spy_words(Ws, H_, code, seeds, incoherent=True, in_seed=None, out_rot=True):
        nets = real_w(Ws, H_, code, seeds, incoherent=incoherent, in_seed=in_seed, out_rot=out_rot)
        words_calls.append((torch.stack(list(Ws)) if len(Ws) == 1 else torch.cat(list(Ws)), code.k, list(seeds),
                            incoherent, in_seed, out_rot,
                            [Q.trellis_states(net.cores["W"].data, code.values) for net in nets]))
        return nets

    C.viterbi, C.ldlq_words = spy_viterbi, spy_words
    try:
        def round_group(rows, bits):
            return Q.word(f"tr{bits}x", W[rows], H, 6100, trellis, in_seed, False)
        Wq, rate, entry = Q.quantize_row_groups(W, groups, round_group, in_seed, True)
    finally:
        C.viterbi, C.ldlq_words = real_v, real_w
    out = {"W": W.float().numpy(), "H": H.float().numpy(), "perm": perm.numpy(), "in_seed": np.array(in_seed),
           "Wq": Wq.float().numpy(), "states": entry["states"].numpy()}
    out["vit_k"] = np.array([c[1] for c in vit_calls])
    out["vit_rows"] = np.array([c[0].shape[0] for c in vit_calls])
    out["vit_T"] = np.array([c[0].shape[1] for c in vit_calls])
    out["vit_X"] = np.concatenate([c[0].reshape(-1).numpy() for c in vit_calls])
    out["vit_start"] = np.concatenate([c[2].numpy() for c in vit_calls])
    out["vit_out"] = np.concatenate([c[3].reshape(-1).numpy() for c in vit_calls])
    for i, (Ws, k, seeds, inc, ins, orot, sts) in enumerate(words_calls):
        out[f"w{i}_W"] = Ws.reshape(-1, Ws.shape[-1]).float().numpy()
        out[f"w{i}_meta"] = np.array([k, seeds[0], int(inc), -1 if ins is None else ins, int(orot)])
        out[f"w{i}_states"] = sts[0].numpy()
    out["words_calls"] = np.array(len(words_calls))
    np.savez_compressed(HERE / "dropin.npz", **out)


def write_small_l_fixture(C, torch):
    """18. Trellises of fewer states (BASELINE config 3's synthetic codebooks: a Lloyd-Max fit to N(0, 1) with
    2^(bits+4) entries, fp16, in the state order trellis_values gives its quantiles): the reference's
    nested.lloyd_max_levels, its viterbi at L = 5..11 (with and without start states), and its ldlq_words with a row
    trellis (L = 6, k = 2) and a column trellis (L = 7, k = 3, T = 64) on those codebooks."""
    from opgraph import nested as NS
    out = {}
    g = torch.Generator().manual_seed(7100)

    def codebook(bits):
        L = bits + 4
        levels = NS.lloyd_max_levels(1 << L).to(torch.float16).double()
        return L, levels[torch.randperm(1 << L, generator=torch.Generator().manual_seed(0))]
    for bits in (1, 2, 3, 4):
        L, v = codebook(bits)
        out[f"codebook_{bits}"] = v.numpy()
    out["lloyd_max_levels_64"] = NS.lloyd_max_levels(64).numpy()
    cases = [("a", 6, 2, 64, 24, True), ("b", 5, 1, 32, 256, False), ("c", 8, 4, 48, 24, True), ("d", 11, 3, 8, 40, False),
             ("e", 7, 3, 40, 320, True)]
    for name, L, k, rows, T, with_start in cases:
        v = torch.randn(1 << L, generator=g, dtype=torch.float64).float().double()
        X = torch.randn(rows, T, generator=g, dtype=torch.float64).float().double()
        start = torch.randint(0, 1 << L, (rows,), generator=g) if with_start else None
        out[f"v{name}_meta"] = np.array([L, k, int(with_start)])
        out[f"v{name}_values"], out[f"v{name}_X"] = v.numpy(), X.numpy()
        if with_start:
            out[f"v{name}_start"] = start.numpy()
        out[f"v{name}_states"] = C.viterbi(X, v, L, k, start=start).numpy()
    real = C.trellis_values
    try:
        L, v = codebook(2)
        C.trellis_values = lambda *a, **kw: v
        code = C.RowTrellisCode(L, 2, T=256, width=16, look=8)
        W = (0.02 * torch.randn(64, 256, generator=g, dtype=torch.float64)).float().double()
        H = calib_H(256, 2048, 7101)
        net = C.ldlq_words([W], H, code, [7102], in_seed=7103, out_rot=False)[0]
        out.update({"row_W": W.float().numpy(), "row_H": H.float().numpy(), "row_Wq": net.matrix(dtype=torch.float64).numpy(),
                    "row_settled": net.cores["W"].data.numpy()})
        L, v = codebook(3)
        C.trellis_values = lambda *a, **kw: v
        code = C.TrellisCode(L, 3, T=64)
        W = (0.02 * torch.randn(128, 64, generator=g, dtype=torch.float64)).float().double()
        H = calib_H(64, 1024, 7104)
        net = C.ldlq_words([W], H, code, [7105])[0]
        out.update({"col_W": W.float().numpy(), "col_H": H.float().numpy(), "col_Wq": net.matrix(dtype=torch.float64).numpy(),
                    "col_settled": net.cores["W"].data.numpy().reshape(128, 64)})
    finally:
        C.trellis_values = real
    np.savez_compressed(HERE / "small_l.npz", **out)


def ast_def():
    import ast
    return ast.FunctionDef


def write_kl_fixture(torch, Q):
    """12. The KL of a probe by the reference's quantize.evaluate (quantize.py:903-920; the formula of
    compiler.py:180-187 and text_kl.py:54-58): a tiny random-init bf16 Llama against a copy with one linear piece
    perturbed (statgen.kl_inputs). Stored with it: both models' final hidden states (the lm_head's input, bf16 bits)
    and the tied lm_head weight, which the KL head kernel takes, and the per-position KL of the same formula."""
    sys.path.insert(0, str(HERE))
    import statgen
    import torch.nn.functional as F
    ref, probe, ids = statgen.kl_inputs()
    res = Q.evaluate(probe, ref, ids, 2)
    grab = {}

    def hook(tag):
        def f(m, a):
            grab.setdefault(tag, []).append(a[0].detach().reshape(-1, a[0].shape[-1]))
        return f
    hs = [ref.lm_head.register_forward_pre_hook(hook("ref")), probe.lm_head.register_forward_pre_hook(hook("probe"))]
    with torch.no_grad():
        lr = F.log_softmax(ref(ids, use_cache=False).logits.float(), -1)
        lp = F.log_softmax(probe(ids, use_cache=False).logits.float(), -1)
    for h in hs:
        h.remove()
    per_pos = (lr.exp() * (lr - lp)).sum(-1).reshape(-1)
    out = {"ids": ids.numpy(), "kl": np.array(res["kl"]), "ppl": np.array(res["ppl"]), "kl_pos": per_pos.numpy(),
           "h_ref": torch.cat(grab["ref"]).view(torch.int16).numpy(),
           "h_probe": torch.cat(grab["probe"]).view(torch.int16).numpy(),
           "E": ref.lm_head.weight.detach().view(torch.int16).numpy()}
    np.savez_compressed(HERE / "kl.npz", **out)


def write_neartie_fixture(C, torch, case: Path):
    """9. A Viterbi near-tie (codes.py:151-181): one 256-step sequence whose best path, in the reference's separately
    rounded fp32 costs, beats another by one ulp at the end — a fused multiply-add in the branch cost picks the other
    one. The input (`case`) is row 131 of batch 1977 of the k = 2, T = 256 e-means table fit (codes.py:187-220) with
    the table of that batch: the fit replayed on a GPU, where a decoder with fused costs first departed from the
    reference's paths. The expected states are the reference's own viterbi of it."""
    d = np.load(case)
    X, v, k = np.asarray(d["X"], dtype=np.float64).reshape(1, -1), np.asarray(d["values"], dtype=np.float64), int(d["k"])
    states = C.viterbi(torch.as_tensor(X), torch.as_tensor(v), 12, k).numpy()
    np.savez_compressed(HERE / "viterbi_neartie.npz", X=X, values=v, k=np.int64(k), states=states)


def write_fit_fixture(C, torch):
    """8. Table fits (codes.py:187-220) by the reference's own trellis_values, short enough for its CPU Viterbi: the
    e-means fit with refine = 1 (16 batches) and two Lloyd steps, for k = 2 and 3 at T = 64."""
    fit = {}
    for k in (2, 3):
        fit[f"ema_k{k}"] = C.trellis_values(12, k, 64, seed=5, refine=1, fit="ema").numpy()
        fit[f"lloyd_k{k}"] = C.trellis_values(12, k, 64, seed=6, refine=2, fit="lloyd").numpy()
    np.savez_compressed(HERE / "fit.npz", **fit)


def write_artifact_fixture(C, Q, CA, torch):
    """7. opgraph-packed-1 (compiler_artifact.py:307-360, :433-442): the reference's own encode_entry of a row-group
    entry (quantize_row_groups' saved form) and decode_rotated of it, with ragged widths and a row count that is not a
    multiple of 32."""
    m, n = 200, 200
    W = (0.02 * torch.randn(m, n, generator=torch.Generator().manual_seed(12), dtype=torch.float64)).float().double()
    H = calib_H(n, 1024, 43)
    perm = torch.randperm(m, generator=torch.Generator().manual_seed(13))
    groups = [{"rows": perm[:40], "bits": 1}, {"rows": perm[40:110], "bits": 2}, {"rows": perm[110:170], "bits": 3},
              {"rows": perm[170:], "bits": 4}]
    trellis = {b: C.RowTrellisCode(12, b, T=256, width=16, look=8) for b in (1, 2, 3, 4)}
    in_seed = 4401

    def round_group(rows, bits):
        return Q.word(f"tr{bits}x", W[rows], H, 4400, trellis, in_seed, False)

    Wq, rate, entry = Q.quantize_row_groups(W, groups, round_group, in_seed, True)
    tensors, meta = CA.encode_entry("w", entry)
    art = {"states": entry["states"].numpy(), "scales": entry["scales"].numpy(), "table": entry["table"].numpy(),
           "in_seed": np.array(in_seed), "signs": tensors["w.signs"], "decoded": CA.decode_rotated(tensors, meta)}
    for i in range(len(groups)):
        art[f"g{i}_rows"] = tensors[f"w.g{i}.rows"]
        art[f"g{i}_codes"] = tensors[f"w.g{i}.codes"]
        art[f"g{i}_scales"] = tensors[f"w.g{i}.scales"]
        art[f"g{i}_bits"] = np.array(meta["groups"][i]["bits"])
    np.savez_compressed(HERE / "artifact.npz", **art)


if __name__ == "__main__":
    main()
