"""Packed trellis rows on B200: the opgraph-packed-1 trellis encoding and the product with packed rows
(liblamq_b200: lamq_pack_trellis, lamq_unpack_trellis, lamq_decode_trellis, lamq_trellis_product,
lamq_trellis_product_groups, lamq_trellis_gemm).

Reference (ShinMegamiBoson/lookatmyquant):
  valid_path, pack_trellis, unpack_trellis      compiler_artifact.py:261-297
  _input_signs                                  compiler_artifact.py:300-304
  encode_entry (state-based row-group entries)  compiler_artifact.py:307-360, grouped_matrix_specs :143-167
  decode_rotated                                compiler_artifact.py:433-442
  the product y = S ⊙ (V[state]·(R_in x))       runtime_mlx/fast_q35.py:69-172 (Metal there); for many vectors
                                                the decode fused into a tcgen05 GEMM (lamq_trellis_gemm)

Tensors live on the device; uint32 words and row maps are held in int32 tensors (the same bits). Invalid input raises
the reference's ValueError messages. There is no host fallback: every entry point runs in liblamq_b200.so.
"""

from __future__ import annotations

import torch

from . import _lib
from ._lib import check, ptr, stream_ptr
from .rotation import Rotation

TABLE_ENTRIES = 4096
STATE_BITS = 12
GEMM_PRODUCT_VECTORS = 64  # from this many input vectors on, the product runs on the tensor cores (lamq_trellis_gemm)


def _dev(t: torch.Tensor) -> torch.device:
    if not t.is_cuda:
        raise RuntimeError("packed trellis tensors must be on a CUDA device")
    return t.device


def _i32(t: torch.Tensor) -> torch.Tensor:
    """uint32 words or row ids held as int32 (the same bits)."""
    if t.dtype in (torch.int32,):
        return t.contiguous()
    if hasattr(torch, "uint32") and t.dtype == torch.uint32:
        return t.contiguous().view(torch.int32)
    return t.to(torch.int64).to(torch.int32).contiguous()


def words_per_row(columns: int, bits: int) -> int:
    return int(_lib.load().lamq_trellis_words_per_row(columns, bits))


def pack_trellis(states: torch.Tensor, bits: int, state_bits: int = STATE_BITS) -> torch.Tensor:
    """compiler_artifact.pack_trellis: rows x n states (a trellis path from state 0 per row) → rows x ⌈n/32⌉·bits
    words (int32 holding uint32)."""
    dev = _dev(states)
    if states.ndim != 2 or states.shape[1] == 0:
        raise ValueError("states are not a row trellis from zero")
    st = states.to(torch.int16) if states.dtype != torch.int16 else states
    if bool(((states < 0) | (states >= 1 << state_bits)).any()):
        raise ValueError("states are not a row trellis from zero")
    st = st.contiguous()
    rows, n = st.shape
    codes = torch.empty(rows, words_per_row(n, bits), dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        check(_lib.load().lamq_pack_trellis(ptr(st), st.stride(0), rows, n, bits, state_bits, ptr(codes), ptr(status),
                                            stream_ptr(dev)), "lamq_pack_trellis")
    if int(status.item()) == _lib.LAMQ_ERR_NOT_PATH:
        raise ValueError("states are not a row trellis from zero")
    return codes


def unpack_trellis(codes: torch.Tensor, bits: int, columns: int, state_bits: int = STATE_BITS) -> torch.Tensor:
    """compiler_artifact.unpack_trellis: the rows x columns states (int16) of packed rows."""
    dev = _dev(codes)
    codes = _i32(codes)
    rows = codes.shape[0]
    if codes.shape != (rows, words_per_row(columns, bits)):
        raise ValueError("code dimensions disagree with width")
    out = torch.empty(rows, columns, dtype=torch.int16, device=dev)
    with torch.cuda.device(dev):
        check(_lib.load().lamq_unpack_trellis(ptr(codes), rows, columns, bits, state_bits, ptr(out), columns,
                                              stream_ptr(dev)), "lamq_unpack_trellis")
    return out


def input_signs(columns: int, seed: int) -> torch.Tensor:
    """compiler_artifact._input_signs: int8 ±1 from torch's CPU generator (the quantizer's exact definition)."""
    u = torch.rand(columns, generator=torch.Generator().manual_seed(int(seed)), dtype=torch.float64)
    return torch.where(u < 0.5, -1, 1).to(torch.int8)


def grouped_matrix_meta(name: str, shape, groups, state_bits: int = STATE_BITS) -> dict:
    """The matrix metadata of compiler_artifact.grouped_matrix_specs for trellis row groups."""
    rows, columns = map(int, shape)
    if sum(int(g["rows"]) for g in groups) != rows:
        raise ValueError("groups must cover the matrix")
    records = []
    for i, g in enumerate(groups):
        m, bits = int(g["rows"]), int(g["bits"])
        if m <= 0 or not 1 <= bits <= 8:
            raise ValueError("empty group or unsupported width")
        records.append({"key": f"{name}.g{i}", "kind": "trellis", "bits": bits, "rows": m, "columns": columns,
                        "padded_columns": (columns + 31) // 32 * 32, "state_bits": state_bits, "start_state": 0})
    return {"kind": "grouped", "shape": [rows, columns], "signs": name + ".signs", "groups": records}


def encode_entry(name: str, entry: dict, signs: torch.Tensor | None = None):
    """compiler_artifact.encode_entry for a state-based row-group entry (quantize_row_groups' saved form: states with
    4096·table_index offsets, fp32 scales, in_seed, concatenated fp32 tables, row_groups). Returns (tensors, meta) with
    the packed codes computed on the device."""
    states = entry["states"]
    if states.ndim != 2:
        raise ValueError("saved entry must be a matrix")
    dev = _dev(states)
    m, n = states.shape
    scales = entry["scales"].to(dev)
    if scales.shape != (m,) or scales.dtype != torch.float32:
        raise ValueError("saved row scales must be fp32, one per row")
    if not bool(torch.isfinite(scales).all()):
        raise ValueError("nonfinite row scales")
    table = entry["table"].to(dev)
    if table.ndim != 1 or table.dtype != torch.float32 or not bool(torch.isfinite(table).all()):
        raise ValueError("saved table must be a finite fp32 vector")
    signs = input_signs(n, entry["in_seed"]) if signs is None else signs.to(torch.int8).cpu()
    if signs.shape != (n,) or not bool(((signs == 1) | (signs == -1)).all()):
        raise ValueError("invalid input signs")
    enc = states.to(torch.int64)
    if table.numel() % TABLE_ENTRIES or bool((enc < 0).any()) or bool((enc >= table.numel()).any()):
        raise ValueError("invalid saved trellis table or states")
    group_ids = enc[:, 0] // TABLE_ENTRIES
    if not bool((enc // TABLE_ENTRIES == group_ids[:, None]).all()):
        raise ValueError("a row crosses table identities")
    if entry.get("row_groups") is None:
        raise ValueError("state-based entries without row_groups: save explicit row_groups metadata")
    tensors = {name + ".signs": signs}
    descriptors, covered = [], []
    for i, g in enumerate(entry["row_groups"]):
        rows = torch.as_tensor(g["rows"], dtype=torch.int64).to(dev)
        bits, ti = int(g["bits"]), int(g["table_index"])
        if rows.ndim != 1 or bool((rows < 0).any()) or bool((rows >= m).any()) or not bool((group_ids[rows] == ti).all()):
            raise ValueError("invalid row group")
        key = f"{name}.g{i}"
        tensors.update({key + ".rows": rows.to(torch.int32), key + ".codes": pack_trellis(enc[rows] - ti * TABLE_ENTRIES, bits),
                        key + ".scales": scales[rows].contiguous(),
                        key + ".table": table[ti * TABLE_ENTRIES:(ti + 1) * TABLE_ENTRIES].contiguous()})
        descriptors.append({"rows": int(rows.numel()), "bits": bits})
        covered.append(rows)
    if not torch.equal(torch.cat(covered).sort().values, torch.arange(m, device=dev)):
        raise ValueError("row groups must cover every row exactly once")
    return tensors, grouped_matrix_meta(name, [m, n], descriptors)


def decode_rotated(tensors: dict, meta: dict) -> torch.Tensor:
    """compiler_artifact.decode_rotated for trellis groups: the fp32 table·scale values before the input transform."""
    m, n = meta["shape"]
    dev = _dev(tensors[meta["groups"][0]["key"] + ".codes"])
    out = torch.empty(m, n, dtype=torch.float32, device=dev)
    lib = _lib.load()
    for g in meta["groups"]:
        if g["kind"] != "trellis":
            raise NotImplementedError("scalar groups are not part of the trellis path")
        key = g["key"]
        codes, rows = _i32(tensors[key + ".codes"]), _i32(tensors[key + ".rows"])
        scales, table = tensors[key + ".scales"].contiguous(), tensors[key + ".table"].contiguous()
        with torch.cuda.device(dev):
            check(lib.lamq_decode_trellis(ptr(codes), rows.numel(), n, g["bits"], g["state_bits"], ptr(scales),
                                          ptr(table), ptr(rows), ptr(out), n, stream_ptr(dev)), "lamq_decode_trellis")
    return out


class TrellisProduct:
    """y = W·x for a packed grouped matrix, W = diag(S)·V[state]·R_in (the product of runtime_mlx/fast_q35.py):
    x is rotated once (R_in x, fp64 through the Kronecker factors, then fp32) and the row groups multiply their packed
    rows with it, all in one launch (lamq_trellis_product_groups; `product_rotated` does the same for every matrix of
    a stage). With GEMM_PRODUCT_VECTORS or more vectors, the rotated input is rounded to bf16 and the groups run as
    one tcgen05 GEMM whose weights are decoded from the packed states into shared memory (lamq_trellis_gemm, fp32
    accumulation): nothing dense is formed."""

    def __init__(self, tensors: dict, meta: dict, device=None):
        self.meta = meta
        self.m, self.n = meta["shape"]
        self.device = torch.device(device or "cuda")
        self.rot = Rotation.from_signs(tensors[meta["signs"]].to(torch.float64), self.device)
        self.groups = []
        for g in meta["groups"]:
            key = g["key"]
            self.groups.append((g, _i32(tensors[key + ".codes"]).to(self.device),
                                _i32(tensors[key + ".rows"]).to(self.device),
                                tensors[key + ".scales"].to(self.device).contiguous(),
                                tensors[key + ".table"].to(self.device).contiguous()))
        self._dense = None

    def rotate(self, x: torch.Tensor) -> torch.Tensor:
        """R_in x for each row of x (nvec x n): fp64 through the factors, then fp32, for the CUDA-core product of few
        vectors; from GEMM_PRODUCT_VECTORS vectors on summed in fp32 and rounded to the GEMM's bf16 operand."""
        x = x.reshape(-1, self.n).to(self.device)
        if x.shape[0] >= GEMM_PRODUCT_VECTORS:
            return self.rot.rows_act(x, torch.bfloat16)
        return self.rot.rows(x.to(torch.float64).contiguous()).to(torch.float32)

    def dense_rotated(self) -> torch.Tensor:
        """decode_rotated as bf16 (cached): V[state]·S before the input transform (a check, not the product path)."""
        if self._dense is None:
            tensors = {}
            for g, codes, rows, scales, table in self.groups:
                tensors.update({g["key"] + ".codes": codes, g["key"] + ".rows": rows, g["key"] + ".scales": scales,
                                g["key"] + ".table": table})
            self._dense = decode_rotated(tensors, self.meta).to(torch.bfloat16)
        return self._dense

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        squeeze = x.ndim == 1
        y = self.rotated(self.rotate(x.reshape(-1, self.n)))
        return y[0] if squeeze else y

    def rotated(self, xr: torch.Tensor) -> torch.Tensor:
        """y = V[state]·S · xr for an input already rotated (R_in x, fp32, nvec × n): matrices that read the same
        input through the same signs (a stage's q/k/v, gate/up) share one rotation."""
        nvec = xr.shape[0]
        y = torch.empty(nvec, self.m, dtype=torch.float32, device=self.device)
        if nvec >= GEMM_PRODUCT_VECTORS:
            _gemm_product([(self, y)], xr)
            return y
        _grouped_product([(self, y)], xr.to(self.device, torch.float32).contiguous())
        return y

    def product_groups(self, y: torch.Tensor) -> list:
        """(lamq_product_group, row group) for each row group of this matrix, writing its rows of y (nvec × m)."""
        return [(_lib.ProductGroup(ptr(codes), rows.numel(), g["bits"], g["state_bits"], ptr(scales), ptr(table),
                                   ptr(rows), ptr(y), y.stride(0)), (g, codes, rows, scales, table))
                for g, codes, rows, scales, table in self.groups]


def _bf16_operand(x: torch.Tensor, device) -> torch.Tensor:
    """x as the GEMM's bf16 operand: 16-byte aligned rows whose length is a multiple of 8 elements (padded)."""
    x = x.to(device, torch.bfloat16)
    n = x.shape[1]
    if x.stride(-1) == 1 and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0:
        return x
    ld = (n + 7) // 8 * 8
    buf = torch.empty(x.shape[0], ld, dtype=torch.bfloat16, device=device)
    buf[:, :n] = x
    return buf[:, :n]


def gemm_groups(groups: list, nvec: int, device, y_bf16: bool = False):
    """lamq_trellis_gemm over `groups` (lamq_gemm_group structures, each with its bf16 input); returns the status
    word (device int32)."""
    status = torch.zeros(1, dtype=torch.int32, device=device)
    if not groups:
        return status
    lib = _lib.load()
    arr = (_lib.GemmGroup * len(groups))(*groups)
    need = lib.lamq_trellis_gemm_workspace_size(arr, len(groups), nvec)
    ws = torch.empty(need, dtype=torch.uint8, device=device) if need else None
    with torch.cuda.device(device):
        check(lib.lamq_trellis_gemm(arr, len(groups), nvec, 1 if y_bf16 else 0, ptr(ws), need, ptr(status),
                                    stream_ptr(device)), "lamq_trellis_gemm")
    return status


def _gemm_product(pairs: list, xr: torch.Tensor):
    """Every row group of the (TrellisProduct, y) pairs times xr (nvec × n) on the tensor cores, one launch."""
    _gemm_layer([(pairs, xr)])


def _gemm_layer(stages: list):
    """[(pairs, xr)]: each stage's (TrellisProduct, y) pairs times its rotated input xr, all in as few launches as
    lamq_trellis_gemm allows (16 groups and 4 inputs a launch)."""
    device = stages[0][0][0][0].device
    nvec = stages[0][1].shape[0]
    groups, keep = [], []
    for pairs, xr in stages:
        x = _bf16_operand(xr, device)
        keep.append(x)
        for prod, y in pairs:
            for g, codes, rows, scales, table in prod.groups:
                groups.append(_lib.GemmGroup(ptr(codes), None, 0, rows.numel(), g["bits"], g["state_bits"],
                                             ptr(scales), ptr(table), ptr(rows), ptr(y), y.stride(0), ptr(x),
                                             x.stride(0), x.shape[1], 0))
    status = gemm_groups(groups, nvec, device)
    st = int(status.item())
    if st:
        _lib.check(st, "lamq_trellis_gemm")


def product_layer(stages: list) -> list:
    """[product_rotated(products, xr) for (products, xr) in stages] with every row group of every stage in one
    tensor-core launch per 16 groups (for many vectors; few vectors take the per-stage grouped product). `stages`:
    [(products, xr)], xr the stage's rotated input (nvec × n), the same nvec for all."""
    if not stages:
        return []
    nvec = stages[0][1].shape[0]
    if nvec < GEMM_PRODUCT_VECTORS:
        return [product_rotated(ps, xr) for ps, xr in stages]
    outs, work = [], []
    for ps, xr in stages:
        ys = [torch.empty(nvec, p.m, dtype=torch.float32, device=p.device) for p in ps]
        outs.append(ys)
        work.append((list(zip(ps, ys)), xr))
    _gemm_layer(work)
    return outs


def _grouped_product(pairs: list, xr: torch.Tensor):
    """Every row group of the (TrellisProduct, y) pairs times xr: the groups of 1-4-bit symbols in one
    lamq_trellis_product_groups call, wider symbols (up to 8 bits) one lamq_trellis_product call each."""
    device, n, nvec = pairs[0][0].device, pairs[0][0].n, xr.shape[0]
    lib = _lib.load()
    narrow, wide = [], []
    for prod, y in pairs:
        for desc, grp in prod.product_groups(y):
            (narrow if desc.k <= 4 else wide).append((desc, grp, y))
    with torch.cuda.device(device):
        if narrow:
            arr = (_lib.ProductGroup * len(narrow))(*[d for d, _, _ in narrow])
            check(lib.lamq_trellis_product_groups(arr, len(narrow), n, ptr(xr), xr.stride(0), nvec,
                                                  stream_ptr(device)), "lamq_trellis_product_groups")
        for _, (g, codes, rows, scales, table), y in wide:
            check(lib.lamq_trellis_product(ptr(codes), rows.numel(), n, g["bits"], g["state_bits"], ptr(scales),
                                           ptr(table), ptr(rows), ptr(xr), xr.stride(0), nvec, ptr(y), y.stride(0),
                                           stream_ptr(device)), "lamq_trellis_product")


def product_rotated(products: list, xr: torch.Tensor) -> list:
    """[p.rotated(xr) for p in products] for matrices that read one rotated input (a stage's q/k/v or gate/up, whose
    entries share their input signs), with every row group of every matrix in one launch. Results are equal to the
    per-matrix calls', bit for bit."""
    if not products:
        return []
    n, device = products[0].n, products[0].device
    if any(p.n != n or p.device != device for p in products):
        raise ValueError("product_rotated: the matrices must share the input width and the device")
    nvec = xr.shape[0]
    ys = [torch.empty(nvec, p.m, dtype=torch.float32, device=device) for p in products]
    if nvec >= GEMM_PRODUCT_VECTORS:
        _gemm_product(list(zip(products, ys)), xr)
    else:
        _grouped_product(list(zip(products, ys)), xr.to(device, torch.float32).contiguous())
    return ys


class TrellisLinear(torch.nn.Module):
    """A linear layer whose weight is a trellis word (codes.TrellisWord: W = R_outᵀ·diag(S)·V[states]·R_in), applied
    without forming W: y = R_outᵀ·(S ⊙ (V[states]·(R_in x))). The input rotation runs through the Kronecker factors,
    the product on the tensor cores straight from the int16 states (lamq_trellis_gemm: bf16 operands, fp32
    accumulation), the output rotation through the factors again; the result is cast to the input's dtype. This is
    how the measure sweep's probe runs its quantized piece (the reference writes the dense word into the model,
    compiler.py:220-229 with quantize.py:332-347)."""

    def __init__(self, word, device=None):
        super().__init__()
        dev = torch.device(device or word.states.device)
        self.word = word
        self.out_features, self.in_features = word.states.shape
        st = word.states.to(dev, torch.int16)
        if st.stride(-1) != 1 or st.stride(0) % 8 or st.data_ptr() % 16 or self.in_features % 8:
            ld = (self.in_features + 7) // 8 * 8
            buf = torch.zeros(self.out_features, ld, dtype=torch.int16, device=dev)
            buf[:, :self.in_features] = st
            st = buf
        self.states = st
        self.scales = word.scales.to(dev, torch.float32).contiguous()
        self.table = torch.as_tensor(word.values).to(dev, torch.float32).contiguous()
        self.L = int(word.L)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        xf = x.reshape(-1, self.in_features)
        xr = self.word.R_in.rows_act(xf, torch.bfloat16) if self.word.R_in is not None else xf
        xb = _bf16_operand(xr, self.states.device)
        nvec = xb.shape[0]
        z = torch.empty(nvec, self.out_features, dtype=torch.float32, device=self.states.device)
        g = _lib.GemmGroup(None, ptr(self.states), self.states.stride(0), self.out_features, 0, self.L,
                           ptr(self.scales), ptr(self.table), None, ptr(z), z.stride(0), ptr(xb), xb.stride(0),
                           self.in_features, 0)
        status = gemm_groups([g], nvec, z.device)
        if self.word.R_out is not None:
            z = self.word.R_out.rows_t_act(z, torch.float32)
        if int(status.item()):
            _lib.check(int(status.item()), "lamq_trellis_gemm")
        return z.to(x.dtype).reshape(*shape[:-1], self.out_features)
