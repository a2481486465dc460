"""fp8 training recipe for the backbone linears (the fp8 variant of the step).

Every backbone linear (q|k|v, output projection, gate|up, down) runs its three
GEMMs on the kind::f8f6f4 tensor cores:

    forward   Y  = X  W^T        X, W in e4m3 (K-major)
    backward  dX = dY W          dY in e5m2, W in e4m3 read MN-major
              dW = dY^T X        dY in e5m2, X in e4m3, both read MN-major

so one row-major 8-bit copy of each tensor serves all three products (the
tcgen05 MN-major operand layout is valid for e4m3 / e5m2).

Each quantised tensor is a *site* with per-tensor delayed scaling: the scale
used in step t is fmax / max(amax history of steps < t) (fmax 448 for e4m3,
57344 for e5m2, history of 16 steps); the cast that quantises the tensor
records its amax, and ``end_step`` pushes those into the histories.  In the
first step (empty histories) each cast first measures its own tensor's amax
("just in time").  Casts are saturating, round-to-nearest-even.

The heads' linears (board, policy, thinking, and the first Linear of the WL
/ D value heads) follow the same recipe with ``heads=`` names: their weight and
logit-gradient sites per head, and one input site per row set -- the pass-1
rows (board head), the pass-2 rows (policy / thinking heads, quantised once
for all pass-2 rows as the reference applies those heads to all of them), and
each value head's gathered rows.  The value heads' second Linear (128 -> 100,
inside the fused value-tail kernel), norms, attention, softmax and the
optimizer stay as in the bf16 step.

The reference has no fp8 path: its linears run in fp16 under torch.autocast
(chessdecoder/train/train.py:168).
"""
from __future__ import annotations

import torch

from . import kernels as K

HIST_LEN = 16
LINEARS = ("qkv", "o", "13", "2")
# head input row sets: pass-1 rows, pass-2 rows, the value heads' gathered rows
HEAD_INPUTS = ("h_causal", "h_prefix", "wl_head.mlp.0", "d_head.mlp.0")


class Fp8Recipe:
    """Scaling state (device arrays, one entry per site) and the per-step fp8
    weight copies of a Backbone."""

    def __init__(self, num_layers: int, device, hist_len: int = HIST_LEN, heads=()):
        self.device = torch.device(device)
        self.hist_len = hist_len
        self.index = {}
        fm = []
        for i in range(num_layers):
            for lin in LINEARS:
                for kind, fmax in (("x", 448.0), ("w", 448.0), ("g", 57344.0)):
                    self.index[(i, lin, kind)] = len(fm)
                    fm.append(fmax)
        # heads: ("head", name, "w" | "g") per head linear, ("head", rows, "x") per input row set
        for name in heads:
            for kind, fmax in (("w", 448.0), ("g", 57344.0)):
                self.index[("head", name, kind)] = len(fm)
                fm.append(fmax)
        for rows in HEAD_INPUTS if heads else ():
            self.index[("head", rows, "x")] = len(fm)
            fm.append(448.0)
        n = len(fm)
        self.n = n
        self.fmax = torch.tensor(fm, device=self.device)
        self.amax = torch.zeros(n, device=self.device)
        self.history = torch.zeros(n, hist_len, device=self.device)
        self.scale = torch.ones(n, device=self.device)
        self.scale_inv = torch.ones(n, device=self.device)
        self.steps = 0  # completed end_step calls
        self.weights = {}  # (layer, linear) -> w8 [N, K]

    def site(self, layer: int, lin: str, kind: str) -> int:
        return self.index[(layer, lin, kind)]

    def head_site(self, name: str, kind: str) -> int:
        return self.index[("head", name, kind)]

    def sinv(self, i: int) -> torch.Tensor:
        return self.scale_inv[i:i + 1]

    def cast(self, x: torch.Tensor, i: int, fmt: int, transpose: bool = False, out=None):
        """8-bit copy [rows, cols] of a 2-D fp32 / bf16 tensor (and, with
        transpose=True, also its [cols, rows] transpose: returns (x8, x8T)).
        out: an 8-bit [rows, cols] destination (row pitch a multiple of 16 B)."""
        rows, cols = x.shape
        if self.steps == 0:
            K.fp8_amax(x, self.amax[i:i + 1])
            K.fp8_scales(self.amax[i:i + 1], None, self.scale[i:i + 1], self.scale_inv[i:i + 1],
                         self.fmax[i:i + 1], mode=1)
            amax = None
        else:
            amax = self.amax[i:i + 1]
        dt = torch.float8_e4m3fn if fmt == K.FP8_E4M3 else torch.float8_e5m2
        x8 = _empty8(rows, cols, dt, self.device) if out is None else out
        xt = _empty8(cols, rows, dt, self.device) if transpose else None
        K.fp8_cast(x, self.scale[i:i + 1], fmt, out=x8, out_t=xt, amax=amax)
        return (x8, xt) if transpose else x8

    def fused(self, i: int, fmt: int, rows: int, cols: int):
        """(out8, q8) for a kernel that writes site i's 8-bit copy itself (the
        cast fused into the producer, amax recorded there), or None in the first
        step, whose just-in-time scale needs the tensor's amax before any cast."""
        if self.steps == 0:
            return None
        dt = torch.float8_e4m3fn if fmt == K.FP8_E4M3 else torch.float8_e5m2
        out = _empty8(rows, cols, dt, self.device)
        return out, (out, fmt, self.scale[i:i + 1], self.amax[i:i + 1])

    def cast_weights(self, layer: int, ws: dict):
        """ws: linear name -> fp32 weight [N, K] (views of the master store)."""
        for lin, w in ws.items():
            self.weights[(layer, lin)] = self.cast(w, self.site(layer, lin, "w"), K.FP8_E4M3)

    def end_step(self):
        K.fp8_scales(self.amax, self.history, self.scale, self.scale_inv, self.fmax, mode=0)
        self.steps += 1

    def state_dict(self):
        return {"amax": self.amax.clone(), "history": self.history.clone(), "scale": self.scale.clone(),
                "scale_inv": self.scale_inv.clone(), "steps": self.steps}


def _empty8(rows: int, cols: int, dtype, device) -> torch.Tensor:
    """[rows, cols] 8-bit tensor whose row pitch is a multiple of 16 bytes (TMA)."""
    pitch = (cols + 15) // 16 * 16
    t = torch.empty(rows, pitch, dtype=dtype, device=device)
    return t[:, :cols]
