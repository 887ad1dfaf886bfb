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

    python tests/golden/make_golden.py --reference /path/to/reference   # part 1
    python tests/golden/make_golden.py --gpu --out gpurun_out/           # part 2
"""
from __future__ import annotations

import argparse
import importlib.util
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


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, default=None)
    ap.add_argument("--gpu", action="store_true")
    ap.add_argument("--out", type=Path, default=HERE)
    args = ap.parse_args()
    if args.gpu:
        make_scaled_mm(args.out)
    else:
        assert args.reference is not None, "--reference <checkout> is required for part 1"
        make_swizzle(args.reference)
