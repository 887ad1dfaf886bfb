"""MoE dispatch and combine around the grouped GEMM (``nvfp4_moe_dispatch`` /
``nvfp4_moe_combine`` in libnvfp4_b200.so).

The reference's grouped GEMM takes each expert's A_g, its permuted scales and
M_g as given (nvfp4_group_gemm/reference.py:39-74, the task tuple of
reference.py:196).  ``dispatch`` produces them from routed tokens on the
device: fp32 activations ``x [T, K]`` and expert choices ``ids [T, topk]``
become one packed NVFP4 buffer whose rows are grouped by expert (stable in
token order), the per-expert scale atoms, and the row / block offsets.
``grouped_inputs`` turns a dispatch plus per-expert weights into the
``(abc, sfasfb, sfasfb_reordered, problem_sizes)`` tuple that
``group_gemm.custom_kernel`` takes, and ``combine`` maps the grouped output
rows back to tokens (weighted sum over each token's choices).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib
from .dual_gemm import on_device


@dataclass
class Dispatch:
    """Device tensors of one dispatch (int32 index arrays, uint8 byte arrays)."""
    packed: torch.Tensor        # [T*topk, K/2]; rows >= row_offsets[E] unused
    sf: torch.Tensor            # flat scale atoms, nvfp4_moe_sf_bytes() bytes
    counts: torch.Tensor        # [E]
    row_offsets: torch.Tensor   # [E+1]
    atom_offsets: torch.Tensor  # [E+1]
    src: torch.Tensor           # [T*topk]: pair index t*topk + j of each permuted row
    dst: torch.Tensor           # [T*topk]: permuted row of each pair, -1 if dropped
    workspace: torch.Tensor
    tokens: int
    topk: int
    k: int
    experts: int


def _alloc(tokens, topk, k, experts, device) -> Dispatch:
    lib = _lib.load()
    pairs = tokens * topk
    i32 = dict(dtype=torch.int32, device=device)
    return Dispatch(
        packed=torch.empty((pairs, k // 2), dtype=torch.uint8, device=device),
        sf=torch.empty(int(lib.nvfp4_moe_sf_bytes(tokens, topk, k, experts)), dtype=torch.uint8,
                       device=device),
        counts=torch.empty(experts, **i32), row_offsets=torch.empty(experts + 1, **i32),
        atom_offsets=torch.empty(experts + 1, **i32), src=torch.empty(pairs, **i32),
        dst=torch.empty(pairs, **i32),
        workspace=torch.empty(int(lib.nvfp4_moe_workspace_bytes(tokens, topk, experts)) // 4,
                              **i32),
        tokens=tokens, topk=topk, k=k, experts=experts)


def dispatch(x: torch.Tensor, expert_ids: torch.Tensor, num_experts: int,
             out: Dispatch | None = None) -> Dispatch:
    """Route ``x`` (CUDA fp32 [T, K], K % 64 == 0) by ``expert_ids`` (int32
    [T] or [T, topk]; ids outside [0, num_experts) are dropped).  ``out``: a
    Dispatch of an earlier call with the same sizes, whose buffers are reused."""
    if x.dim() != 2 or x.dtype != torch.float32 or not x.is_cuda:
        raise ValueError("x must be a CUDA float32 tensor [tokens, K]")
    ids = expert_ids if expert_ids.dim() == 2 else expert_ids.unsqueeze(1)
    if ids.dim() != 2 or ids.shape[0] != x.shape[0] or ids.dtype != torch.int32:
        raise ValueError("expert_ids must be int32 [tokens] or [tokens, topk]")
    if ids.device != x.device:
        raise ValueError("x and expert_ids must be on the same device")
    tokens, k = x.shape
    topk = ids.shape[1]
    if k % 64:
        raise ValueError(f"K={k} must be a multiple of 64")
    x, ids = x.contiguous(), ids.contiguous()
    if out is None:
        out = _alloc(tokens, topk, k, num_experts, x.device)
    elif (out.tokens, out.topk, out.k, out.experts) != (tokens, topk, k, num_experts) or \
            out.packed.device != x.device:
        raise ValueError("out does not match: pass a Dispatch made for the same sizes")
    d = out
    lib = _lib.load()
    _lib.check(on_device(x.device, lambda st: lib.nvfp4_moe_dispatch(
        x.data_ptr(), ids.data_ptr(), tokens, topk, k, num_experts, d.packed.data_ptr(),
        d.sf.data_ptr(), d.counts.data_ptr(), d.row_offsets.data_ptr(),
        d.atom_offsets.data_ptr(), d.src.data_ptr(), d.dst.data_ptr(), d.workspace.data_ptr(),
        d.workspace.numel() * 4, st)))
    return d


def expert_operands(d: Dispatch, counts=None):
    """Per expert: (a [M, K/2, 1] float4_e2m1fn_x2, sfa_perm [32, 4, ceil(M/128),
    4, K/64, 1] float8_e4m3fn, M) as views into the dispatch buffers.  Reads
    the counts back to the host (a synchronisation) unless ``counts`` (a list
    of ints) is given."""
    counts = [int(v) for v in (d.counts.tolist() if counts is None else counts)]
    ka = d.k // 64
    ops, row, blk = [], 0, 0
    for m in counts:
        rb = -(-m // 128)
        a = d.packed[row:row + m].view(torch.float4_e2m1fn_x2).unsqueeze(-1)
        atoms = d.sf[blk * ka * 512:(blk + rb) * ka * 512].view(1, rb, ka, 32, 4, 4)
        sfa = atoms.permute(3, 4, 1, 5, 2, 0).view(torch.float8_e4m3fn)
        ops.append((a, sfa, m))
        row += m
        blk += rb
    return ops


def grouped_inputs(d: Dispatch, weights, c_all: torch.Tensor, counts=None):
    """The grouped-GEMM task tuple for C_e = A_e . W_eᵀ over the experts with
    tokens.  ``weights``: per expert (w [N, K/2, 1] float4_e2m1fn_x2, sfw_perm
    [32, 4, ceil(N/128), 4, K/64, 1]); ``c_all``: fp16 [T*topk, N], expert e's
    output lands in rows [row_offsets[e], +M_e).  Returns (data, experts) with
    ``experts`` the expert index of each group in ``data``."""
    ops = expert_operands(d, counts)
    n = c_all.shape[1]
    abc, sfab, sfab_perm, sizes, which = [], [], [], [], []
    row = 0
    for e, ((a, sfa, m), (w, sfw)) in enumerate(zip(ops, weights)):
        if m > 0:
            abc.append((a, w, c_all[row:row + m].unsqueeze(-1)))
            sfab.append((None, None))          # plain scales: unused by the kernels
            sfab_perm.append((sfa, sfw))
            sizes.append((m, n, d.k, 1))
            which.append(e)
        row += m
    return (abc, sfab, sfab_perm, sizes), which


class ExpertWeights:
    """Per-expert NVFP4 weights for :func:`grouped_gemm`: ``w[e]`` = (b [N, K/2, 1]
    float4_e2m1fn_x2 (or uint8 [N, K/2]), sfb_perm [32, 4, ceil(N/128), 4, K/64, 1]),
    all on one device.  The pointer arrays for the C call are built once."""

    def __init__(self, w):
        self.w = list(w)
        if not self.w:
            raise ValueError("no experts")
        b0 = self.w[0][0]
        self.n, self.k = int(b0.shape[0]), int(b0.shape[1]) * 2
        arr = ctypes.c_void_p * len(self.w)
        for i, (b, sfb) in enumerate(self.w):
            if tuple(b.shape[:2]) != (self.n, self.k // 2) or not b.is_cuda:
                raise ValueError(f"expert {i}: weights must be CUDA [{self.n}, {self.k // 2}(, 1)]")
            if b.stride(0) != self.k // 2 or b.stride(1) != 1 or b.device != b0.device:
                raise ValueError(f"expert {i}: weights must be row-major [N][K/2] on {b0.device}")
            rn, rk = -(-self.n // 128), self.k // 64
            if sfb.numel() != rn * rk * 512 or sfb.device != b0.device:
                raise ValueError(f"expert {i}: scales must hold {rn * rk * 512} bytes on {b0.device}")
        self.b_ptrs = arr(*[b.data_ptr() for b, _ in self.w])
        self.sfb_ptrs = arr(*[s.data_ptr() for _, s in self.w])

    def __len__(self):
        return len(self.w)


def grouped_gemm(d: Dispatch, weights: ExpertWeights, c_all: torch.Tensor) -> torch.Tensor:
    """C_e = A_e . W_eᵀ for every expert straight from the dispatch's device
    sizes (no host synchronisation): expert e's output lands in rows
    [row_offsets[e], +counts[e]) of ``c_all`` (fp16 [T*topk, N])."""
    if len(weights) != d.experts or weights.k != d.k:
        raise ValueError(f"weights are for {len(weights)} experts x K={weights.k}, "
                         f"dispatch has {d.experts} x K={d.k}")
    rows = d.tokens * d.topk
    if (c_all.dtype != torch.float16 or tuple(c_all.shape) != (rows, weights.n)
            or not c_all.is_contiguous() or c_all.device != d.packed.device):
        raise ValueError(f"c_all must be a contiguous float16 [{rows}, {weights.n}] tensor "
                         f"on {d.packed.device}")
    lib = _lib.load()
    _lib.check(on_device(c_all.device, lambda st: lib.nvfp4_moe_grouped_gemm(
        d.packed.data_ptr(), rows, d.sf.data_ptr(), d.counts.data_ptr(), d.row_offsets.data_ptr(),
        d.atom_offsets.data_ptr(), weights.b_ptrs, weights.sfb_ptrs, d.experts, weights.n, d.k,
        c_all.data_ptr(), st)))
    return c_all


def combine(c_all: torch.Tensor, d: Dispatch, weights: torch.Tensor | None = None,
            out: torch.Tensor | None = None) -> torch.Tensor:
    """out[t] = sum_j weights[t, j] * c_all[dst[t*topk + j]] (fp32 [T, N]);
    ``weights`` fp32 [T] or [T, topk], None for all ones."""
    if c_all.dim() != 2 or c_all.dtype != torch.float16 or not c_all.is_contiguous():
        raise ValueError("c_all must be a contiguous float16 tensor [rows, N]")
    n = c_all.shape[1]
    if weights is not None:
        weights = weights.reshape(d.tokens, d.topk)
        if weights.dtype != torch.float32 or weights.device != c_all.device:
            raise ValueError("weights must be float32 on c_all's device")
        weights = weights.contiguous()
    if out is None:
        out = torch.empty((d.tokens, n), dtype=torch.float32, device=c_all.device)
    elif tuple(out.shape) != (d.tokens, n) or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError("out must be a contiguous float32 tensor [tokens, N]")
    lib = _lib.load()
    _lib.check(on_device(c_all.device, lambda st: lib.nvfp4_moe_combine(
        c_all.data_ptr(), c_all.shape[0], d.dst.data_ptr(),
        weights.data_ptr() if weights is not None else None,
        d.tokens, d.topk, n, out.data_ptr(), st)))
    return out
