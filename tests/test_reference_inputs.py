"""CPU: the restated reference generators make the reference's own inputs.

``inputs.reference_dual_input`` / ``reference_group_input`` restate the
reference's ``generate_input`` (nvfp4_dual_gemm/reference.py:80-196,
nvfp4_group_gemm/reference.py:126-196) call for call.  The fixture
``golden/reference_inputs_golden.json`` holds SHA-256 digests of every tensor
the reference's own generators return when their "cuda" tensors are made on
the CPU (tests/golden/make_golden.py, part 3).  Run on the CPU, the
restatement must reproduce every digest: it draws the same random numbers in
the same order from the same generators, so on a GPU it yields the tensors
the reference's harness would hand to ``custom_kernel`` for the same seed.
"""
import importlib.util
import json
from pathlib import Path

import pytest
import torch

from nvfp4_b200 import inputs as I

HERE = Path(__file__).resolve().parent
GOLDEN = json.loads((HERE / "golden" / "reference_inputs_golden.json").read_text())


def _golden_module():
    spec = importlib.util.spec_from_file_location("make_golden", HERE / "golden" / "make_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


MG = _golden_module()


@pytest.mark.parametrize("entry", GOLDEN["dual"], ids=lambda e: "x".join(map(str, e["case"])))
def test_dual_generator_matches_reference(entry):
    m, n, k, l, seed = entry["case"]
    got = MG.input_digests("dual", I.reference_dual_input(m, n, k, l, seed, device="cpu"))
    assert got == entry["digests"]


@pytest.mark.parametrize("entry", GOLDEN["group"], ids=lambda e: f"g{e['case'][3]}-s{e['case'][4]}")
def test_group_generator_matches_reference(entry):
    m, n, k, g, seed = entry["case"]
    got = MG.input_digests("group", I.reference_group_input(m, n, k, g, seed, device="cpu"))
    assert got == entry["digests"]


def test_digests_see_a_changed_seed():
    m, n, k, l, seed = GOLDEN["dual"][0]["case"]
    got = MG.input_digests("dual", I.reference_dual_input(m, n, k, l, seed + 1, device="cpu"))
    assert got["a"] != GOLDEN["dual"][0]["digests"]["a"]


def test_dual_permuted_scales_hold_the_plain_scales():
    d = I.reference_dual_input(100, 136, 320, 1, 5, device="cpu")
    for plain, perm in zip(d[3:6], d[6:9]):
        mn, sf_k = plain.shape[0], plain.shape[1]
        assert torch.equal(MG._valid_scales(perm, mn, sf_k), plain.view(torch.uint8))
