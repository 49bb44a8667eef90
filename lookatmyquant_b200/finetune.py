"""The fine-tuning's trellis parts on B200: re-picking a trellis-coded matrix's paths along its summed gradient, and
rounding real weights back onto a build's row-trellis form (ShinMegamiBoson/lookatmyquant, finetune_lib.py:84-150
`path_bits`, `TrellisCoded`; :203-263 `RowPath`, `rotated_moment`, `rounded`).

`TrellisCoded` holds W = diag(S)·T[state]·R with the matrix's own 4096-entry table T and row scales S as parameters;
`take_gradient` forms their gradients from ∂loss/∂W by hand (and sums each entry's gradient when the paths may move),
and `repick` takes one proximal step: each row's new path is the trellis path nearest c − η·g (c the current values),
a Viterbi from state 0 on the device (lamq_viterbi, states identical to the reference's). `rounded` is a build's
rounding of W under a stage's rotated statistics: the fused row-trellis LDLQ sweep (lamq_ldlq_rowtrellis) per row
group with the group's own table, then the reference's scale refit ((x·gH)/(g·gH) per row, gH on the fp64 tensor
cores). Rotations run through the Hadamard factors (lamq_rht_rows) in fp64 (the reference's FastRHT runs them in
fp32; the products are rounded to fp32 where it keeps fp32).
"""

from __future__ import annotations

import torch

from . import codes
from .layer import sweep_rows
from .linalg import gemm
from .rotation import Rotation

L_TRELLIS = 12  # state bits of every trellis in the builds (finetune_lib.py:77)


def path_bits(states: torch.Tensor) -> int:
    """k, the bits per entry of a row trellis's paths: each state is the one before shifted k bits, from state 0
    (finetune_lib.py:80-86)."""
    s = states.long()
    for k in range(1, L_TRELLIS):
        if bool((s[:, 0] < (1 << k)).all()) and bool(((s[:, 1:] >> k) == (s[:, :-1] & ((1 << (L_TRELLIS - k)) - 1))).all()):
            return k
    raise ValueError("states that are not paths through a row trellis")


class TrellisCoded(torch.nn.Module):
    """A trellis-coded matrix as a build stores it (finetune_lib.py:89-150): `entry` = {"states" (rows x n int),
    "scales" (rows fp32), "table" (4096 fp32), "in_seed"}. W = diag(S)·T[state]·R, R = rht(n, in_seed). With `move`,
    each entry sums its gradient and repick() moves each row along it; otherwise the states stay."""

    def __init__(self, entry: dict, move: bool = False, device=None, rotations: dict | None = None):
        super().__init__()
        dev = codes._dev(device)
        self.register_buffer("states", torch.as_tensor(entry["states"]).to(dev, torch.int16))
        n = self.states.shape[1]
        rotations = {} if rotations is None else rotations
        key = (n, int(entry["in_seed"]))
        if key not in rotations:
            rotations[key] = Rotation(n, int(entry["in_seed"]), dev)
        self.R = rotations[key]
        self.log_s = torch.nn.Parameter(torch.as_tensor(entry["scales"]).to(dev, torch.float32).clamp_min(1e-12).log())
        self.table = torch.nn.Parameter(torch.as_tensor(entry["table"]).to(dev, torch.float32).clone())
        self.k = None
        if move:
            self.k = path_bits(self.states)
            self.register_buffer("acc", torch.zeros(self.states.shape, device=dev))

    def scales(self) -> torch.Tensor:
        return self.log_s.exp()[:, None]

    def matrix(self) -> torch.Tensor:
        """W = diag(S)·T[state]·R (fp32)."""
        Q = self.scales() * self.table[self.states.long()]
        return self.R.rows_t(Q.double()).float()

    @torch.no_grad()
    def take_gradient(self, dW: torch.Tensor):
        """The gradients of the row scales and the table from ∂loss/∂W (finetune_lib.py:118-130), and with `move`
        each entry's summed gradient."""
        g = self.R.rows(dW.double()).float() * self.scales()
        idx = self.states.long()
        gv = g * self.table[idx]
        self.log_s.grad = gv.sum(1)
        self.table.grad = torch.zeros_like(self.table).index_add_(0, idx.flatten(), g.flatten())
        if self.k is not None:
            self.acc += g

    @torch.no_grad()
    def nearest(self, eta: float) -> torch.Tensor:
        """Each row's path for one proximal step on the summed gradient g (finetune_lib.py:132-138): the path nearest
        c − η·g over paths from state 0, c the current values (int16 states)."""
        if self.k is None:
            raise ValueError("the paths move only with move=True")
        c = self.table.detach()[self.states.long()]
        X = c - eta * self.acc
        start = torch.zeros(len(c), dtype=torch.long, device=c.device)
        return codes.viterbi(X, self.table.detach(), L_TRELLIS, self.k, start=start).to(torch.int16)

    @torch.no_grad()
    def repick(self, eta: float) -> float:
        """Takes the step (finetune_lib.py:140-145); returns the share of entries whose state changed."""
        new = self.nearest(eta)
        changed = float((new != self.states).float().mean())
        self.states.copy_(new)
        self.acc.zero_()
        return changed


class RowPath:
    """A build's row trellis (codes.RowTrellisCode with width 16, look 8: each row one path from state 0) with the
    table the build stored (finetune_lib.py:207-222)."""

    def __init__(self, table, k: int, width: int = 16, look: int = 8):
        self.values = torch.as_tensor(table).double().cpu()
        self.k, self.width, self.look = k, width, look


def rotated_moment(H: torch.Tensor, R: Rotation) -> torch.Tensor:
    """The input statistics in the rotated basis, R·H·Rᵀ, symmetrised (finetune_lib.py:228-233)."""
    Hr = R.conj(H.double())
    return (Hr + Hr.T) / 2


@torch.no_grad()
def rounded(W: torch.Tensor, R: Rotation, groups: list, scale: torch.Tensor, env, rows: torch.Tensor | None = None):
    """P(W) as a build rounds, and each entry's state in its group's table (finetune_lib.py:236-263): block LDLQ under
    env (the stage's rotated statistics: its .H, .U and .dead) with each row group (rows, bits per entry, RowPath)
    through its row trellis in units of `scale`, which is then refitted under the same statistics in place
    (scale = (x·gH)/(g·gH) per row, g the settled values, clamped at 1e-12). With `rows` only those rows are rounded
    (rows do not interact) and their stored rows and states come back in that order. Returns (P(W) fp32, int16 states
    on the CPU)."""
    dev = W.device
    X = R.rows((W if rows is None else W[rows]).double()).float().double()
    where = None
    if rows is not None:
        rows = rows.to(dev)
        where = torch.full((W.shape[0],), -1, dtype=torch.long, device=dev)
        where[rows] = torch.arange(len(rows), device=dev)
    Q = torch.empty_like(X)
    states = torch.empty(X.shape, dtype=torch.int16)
    H = env.H.to(dev, torch.float64)
    for g_rows, k, code in groups:
        g_rows = torch.as_tensor(g_rows).to(dev)
        mine = g_rows if where is None else g_rows[where[g_rows] >= 0]
        if not len(mine):
            continue
        at = mine if where is None else where[mine]
        x, S = X[at].contiguous(), scale[mine].to(dev).double()
        tables = torch.zeros(4, 1 << L_TRELLIS, dtype=torch.float64, device=dev)
        tables[k - 1] = code.values.to(dev)
        st, got = sweep_rows(x, S, env, torch.full((len(at),), k, dtype=torch.uint8, device=dev), tables)
        gH = gemm(got, H)
        scale[mine] = ((x * gH).sum(1) / (got * gH).sum(1).clamp_min(1e-30)).clamp_min(1e-12).to(scale.dtype).to(
            scale.device)
        Q[at] = got
        states[at.cpu()] = st.cpu()
    units = scale if rows is None else scale[rows.to(scale.device)]
    return R.rows_t((units.to(dev).double()[:, None] * Q.float().double())).float(), states
