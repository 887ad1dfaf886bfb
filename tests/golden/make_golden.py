"""Generate the golden fixtures in this folder.

Part 1 (CPU, needs the reference checkout): imports the reference's own
``to_blocked`` (nvfp4_group_gemm/reference.py:14-36, and the dual copy at
nvfp4_dual_gemm/reference.py:13-24) and records its output for a set of seeded
scale matrices -> ``swizzle_golden.npz``.  The reference's permuted-layout
builder (``create_reordered_scale_factor_tensor``,
nvfp4_group_gemm/reference.py:80-123) hard-codes ``device='cuda'``; its index
math (``mm32, mm4, mm, kk4, kk``, lines 111-121) is executed here on CPU with
the same torch advanced-indexing statement to produce the permuted images.

Part 2 (GPU box, ``--gpu``): runs ``torch._scaled_mm`` exactly as the
reference's ``ref_kernel`` does (nvfp4_dual_gemm/reference.py:50-76,
nvfp4_group_gemm/reference.py:56-72) on small seeded inputs and stores inputs
and outputs -> ``scaled_mm_golden.npz``.

Part 3 (CPU, needs the reference checkout): runs the reference's own
``generate_input`` (nvfp4_dual_gemm/reference.py:80-196,
nvfp4_group_gemm/reference.py:126-196) with every ``device="cuda"`` it names
redirected to the CPU, and records a SHA-256 digest of each tensor it returns
-> ``reference_inputs_golden.json``.  ``nvfp4_b200.inputs.reference_dual_input``
/ ``reference_group_input`` restate those generators call for call; run on the
CPU they must reproduce the digests, which shows they make the same RNG calls
in the same order (on a GPU both then draw from the CUDA generator).

    python tests/golden/make_golden.py --reference /path/to/reference   # parts 1 and 3
    python tests/golden/make_golden.py --gpu --out <out-dir>/           # part 2
"""
from __future__ import annotations

import argparse
import contextlib
import hashlib
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

SWIZZLE_CASES = [  # (rows, cols) of a [rows, K/16] scale matrix
    (128, 4), (256, 16), (96, 8), (40, 16), (200, 12), (128, 64), (1, 4), (300, 20),
]


def _load_reference_module(ref_root: Path, sub: str):
    path = ref_root / sub / "reference.py"
    # reference.py imports `task` and `utils` from its own folder
    sys.path.insert(0, str(path.parent))
    try:
        spec = importlib.util.spec_from_file_location(f"ref_{sub}", path)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
    finally:
        sys.path.pop(0)
        for name in ("task", "utils"):
            sys.modules.pop(name, None)
    return mod


def make_swizzle(ref_root: Path):
    grp = _load_reference_module(ref_root, "nvfp4_group_gemm")
    dual = _load_reference_module(ref_root, "nvfp4_dual_gemm")
    out = {}
    g = torch.Generator().manual_seed(20240)
    for idx, (rows, cols) in enumerate(SWIZZLE_CASES):
        sf = torch.randint(0, 256, (rows, cols), dtype=torch.uint8, generator=g)
        out[f"sf_{idx}"] = sf.numpy()
        # reference to_blocked (zero-padding variant) on CPU
        blocked = grp.to_blocked(sf.view(torch.float8_e4m3fn)).view(torch.uint8)
        out[f"blocked_{idx}"] = blocked.numpy()
        if rows % 128 == 0 and cols % 4 == 0:  # the dual variant requires full atoms
            out[f"blocked_dual_{idx}"] = dual.to_blocked(sf.view(torch.float8_e4m3fn)) \
                .view(torch.uint8).numpy()
        # permuted image with the reference's own index statement
        # (nvfp4_group_gemm/reference.py:84-121), run on CPU
        l, mn, sf_k = 1, rows, cols
        atom_m, atom_k = (32, 4), 4
        mma_shape = (l, -(-mn // 128), -(-sf_k // atom_k), atom_m[0], atom_m[1], atom_k)
        reordered = torch.zeros(mma_shape, dtype=torch.uint8).permute(3, 4, 1, 5, 2, 0)
        ref3 = sf.unsqueeze(-1)
        i_g, j_g, b_g = torch.meshgrid(torch.arange(mn), torch.arange(sf_k), torch.arange(l),
                                       indexing="ij")
        mm, mm32, mm4 = i_g // 128, i_g % 32, (i_g % 128) // 32
        kk, kk4 = j_g // atom_k, j_g % atom_k
        reordered[mm32, mm4, mm, kk4, kk, b_g] = ref3[i_g, j_g, b_g]
        # memory image: contiguous (l, rest_mn, rest_k, 32, 4, 4)
        out[f"perm_{idx}"] = reordered.permute(5, 2, 4, 0, 1, 3).contiguous().numpy()
    np.savez_compressed(HERE / "swizzle_golden.npz", **out)
    print("wrote", HERE / "swizzle_golden.npz")


GEMM_CASES = [  # (m, n, k, seed)
    (128, 128, 256, 11), (256, 384, 512, 12), (96, 208, 768, 13),
]


def make_scaled_mm(out_dir: Path):
    """Run on a B200: record torch._scaled_mm results on seeded random codes."""
    assert torch.cuda.is_available()
    from torch.nn.functional import silu  # noqa: F401
    out = {}
    for idx, (m, n, k, seed) in enumerate(GEMM_CASES):
        g = torch.Generator().manual_seed(seed)
        a = torch.randint(0, 256, (m, k // 2), dtype=torch.uint8, generator=g)
        b1 = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, generator=g)
        b2 = torch.randint(0, 256, (n, k // 2), dtype=torch.uint8, generator=g)
        # finite e2m1 codes are all 16 nibbles; scales: finite e4m3 in [2^-6, 4)
        mk_sf = lambda r: (torch.rand((r, k // 16), generator=g) * 4 + 2 ** -6) \
            .to(torch.float8_e4m3fn).view(torch.uint8)
        sfa, sfb1, sfb2 = mk_sf(m), mk_sf(n), mk_sf(n)

        def blocked(sf):
            rows, cols = sf.shape
            rb, cb = -(-rows // 128), -(-cols // 4)
            p = torch.zeros((rb * 128, cb * 4), dtype=torch.uint8)
            p[:rows, :cols] = sf
            return p.view(rb, 128, cb, 4).permute(0, 2, 1, 3).reshape(-1, 4, 32, 4) \
                .transpose(1, 2).reshape(-1).view(torch.float8_e4m3fn).cuda()

        fa = a.cuda().view(torch.float4_e2m1fn_x2)
        r1 = torch._scaled_mm(fa, b1.cuda().view(torch.float4_e2m1fn_x2).t(), blocked(sfa),
                              blocked(sfb1), bias=None, out_dtype=torch.float32)
        r2 = torch._scaled_mm(fa, b2.cuda().view(torch.float4_e2m1fn_x2).t(), blocked(sfa),
                              blocked(sfb2), bias=None, out_dtype=torch.float32)
        h = torch._scaled_mm(fa, b1.cuda().view(torch.float4_e2m1fn_x2).t(), blocked(sfa),
                             blocked(sfb1), bias=None, out_dtype=torch.float16)
        out.update({f"a_{idx}": a.numpy(), f"b1_{idx}": b1.numpy(), f"b2_{idx}": b2.numpy(),
                    f"sfa_{idx}": sfa.numpy(), f"sfb1_{idx}": sfb1.numpy(),
                    f"sfb2_{idx}": sfb2.numpy(), f"r1_{idx}": r1.cpu().numpy(),
                    f"r2_{idx}": r2.cpu().numpy(), f"h16_{idx}": h.cpu().numpy(),
                    f"dual_{idx}": (torch.nn.functional.silu(r1) * r2).half().cpu().numpy()})
    out_dir.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(out_dir / "scaled_mm_golden.npz", **out)
    print("wrote", out_dir / "scaled_mm_golden.npz")


# (m, n, k, l, seed) / (m list, n list, k list, g, seed): ragged rows, L = 2,
# a K that leaves a partial 4-block column of scale atoms, the task seeds
DUAL_INPUT_CASES = [(128, 256, 256, 1, 1111), (256, 384, 512, 2, 1153), (100, 136, 320, 1, 1195)]
GROUP_INPUT_CASES = [([96, 128], [128, 256], [256, 512], 2, 1111),
                     ([40, 56, 200], [512, 384, 136], [256, 320, 512], 3, 1153)]


def _u8(t: torch.Tensor) -> torch.Tensor:
    """Logical-order bytes (same shape for 1-byte types, flat otherwise)."""
    t = t.cpu()
    if t.element_size() == 1:
        return t.view(torch.uint8).contiguous()
    return t.contiguous().reshape(-1).view(torch.uint8)


def _digest(t: torch.Tensor) -> str:
    return hashlib.sha256(_u8(t).numpy().tobytes()).hexdigest()


def _valid_scales(perm: torch.Tensor, mn: int, sf_k: int) -> torch.Tensor:
    """[mn, sf_k, l] scales read back out of a permuted [32,4,rm,4,rk,l] tensor."""
    r = torch.arange(mn)[:, None]
    j = torch.arange(sf_k)[None, :]
    u = _u8(perm)
    return u[r % 32, (r % 128) // 32, r // 128, j % 4, j // 4, :]


def input_digests(kind: str, data) -> dict:
    """Digests of every tensor of a task tuple.  Dual permuted scale tensors
    are digested over their written entries only: the reference leaves their
    padding uninitialised."""
    if kind == "dual":
        names = ["a", "b1", "b2", "sfa", "sfb1", "sfb2", "sfa_perm", "sfb1_perm", "sfb2_perm", "c"]
        out = {}
        for i, (name, t) in enumerate(zip(names, data)):
            if name.endswith("_perm"):
                plain = data[i - 3]
                t = _valid_scales(t, plain.shape[0], plain.shape[1])
            out[name] = _digest(t)
        return out
    abc, sfab, perm, sizes = data
    out = {"sizes": [list(s) for s in sizes]}
    for g, ((a, b, c), (sa, sb), (pa, pb)) in enumerate(zip(abc, sfab, perm)):
        for name, t in (("a", a), ("b", b), ("c", c), ("sfa", sa), ("sfb", sb),
                        ("sfa_perm", pa), ("sfb_perm", pb)):
            out[f"{name}_{g}"] = _digest(t)
    return out


@contextlib.contextmanager
def cuda_redirected_to_cpu():
    """Every tensor a function asks for on "cuda" is made on the CPU instead
    (factory calls with device=..., .cuda(), .to("cuda"))."""
    def redirect(kw):
        d = kw.get("device")
        if d is not None and torch.device(d).type == "cuda":
            kw["device"] = "cpu"
        return kw

    saved = {}
    for name in ("randint", "randn", "rand", "empty", "arange", "zeros"):
        saved[name] = getattr(torch, name)
        setattr(torch, name, lambda *a, _f=saved[name], **kw: _f(*a, **redirect(kw)))
    to0, cuda0 = torch.Tensor.to, torch.Tensor.cuda

    def to(self, *a, **kw):
        if a and isinstance(a[0], (str, torch.device)) and torch.device(a[0]).type == "cuda":
            return self
        return to0(self, *a, **kw)

    torch.Tensor.to = to
    torch.Tensor.cuda = lambda self, *a, **kw: self
    try:
        yield
    finally:
        for name, f in saved.items():
            setattr(torch, name, f)
        torch.Tensor.to, torch.Tensor.cuda = to0, cuda0


def make_reference_inputs(ref_root: Path):
    dual = _load_reference_module(ref_root, "nvfp4_dual_gemm")
    grp = _load_reference_module(ref_root, "nvfp4_group_gemm")
    out = {"dual": [], "group": []}
    with cuda_redirected_to_cpu():
        for case in DUAL_INPUT_CASES:
            out["dual"].append({"case": list(case),
                                "digests": input_digests("dual", dual.generate_input(*case))})
        for case in GROUP_INPUT_CASES:
            out["group"].append({"case": [list(case[0]), list(case[1]), list(case[2]), case[3],
                                          case[4]],
                                 "digests": input_digests("group", grp.generate_input(*case))})
    out["torch"] = torch.__version__
    path = HERE / "reference_inputs_golden.json"
    path.write_text(json.dumps(out, indent=1) + "\n")
    print("wrote", path)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=None)
    ap.add_argument("--gpu", action="store_true")
    ap.add_argument("--out", type=Path, default=HERE)
    args = ap.parse_args()
    if args.gpu:
        make_scaled_mm(args.out)
    else:
        assert args.reference is not None, "--reference <checkout> is required for parts 1, 3"
        make_swizzle(args.reference)
        make_reference_inputs(args.reference)
