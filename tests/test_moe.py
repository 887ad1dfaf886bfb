"""MoE dispatch / combine (the routing step in front of the grouped GEMM and
the un-permute behind it).

The reference has no router (its grouped GEMM takes each group's A_g as
given, nvfp4_group_gemm/reference.py:39-74), so the dispatch is pinned to its
own definition: the oracle restatement (oracle.moe_route / moe_dispatch /
moe_combine) is checked here against plain-Python loops, and the CUDA path
against the oracle bit-exactly (all integer / byte results, and a combine
whose fp32 arithmetic is reproduced operation by operation).  The MoE layer
test chains dispatch -> grouped GEMM -> combine against the oracle at the
GEMM tolerance (rtol = atol = 1e-2).
"""
import numpy as np
import pytest
import torch

from oracle import nvfp4_oracle as O


def _loop_route(ids, experts):
    """Plain-Python restatement: walk pairs in order, append to the expert's list."""
    ids = [int(v) for v in np.asarray(ids).reshape(-1)]
    lists = [[] for _ in range(experts)]
    for p, e in enumerate(ids):
        if 0 <= e < experts:
            lists[e].append(p)
    src = [p for lst in lists for p in lst]
    dst = [-1] * len(ids)
    for r, p in enumerate(src):
        dst[p] = r
    counts = [len(lst) for lst in lists]
    return counts, src, dst


@pytest.mark.parametrize("t,topk,e,seed", [(50, 1, 4, 0), (37, 2, 5, 1), (200, 3, 16, 2), (1, 1, 1, 3)])
def test_oracle_route_matches_loop(t, topk, e, seed):
    rng = np.random.default_rng(seed)
    ids = rng.integers(-2, e + 2, size=(t, topk))        # some dropped ids on both sides
    counts, row_off, atom_off, src, dst = O.moe_route(ids, e)
    c2, s2, d2 = _loop_route(ids, e)
    assert counts.tolist() == c2 and src.tolist() == s2 and dst.tolist() == d2
    assert row_off.tolist() == [0] + np.cumsum(c2).tolist()
    assert atom_off.tolist() == [0] + np.cumsum([-(-c // 128) for c in c2]).tolist()


def test_oracle_dispatch_layout():
    rng = np.random.default_rng(5)
    t, k, e = 300, 128, 3
    x = rng.standard_normal((t, k)).astype(np.float32)
    ids = rng.integers(0, e, size=(t, 1))
    (counts, row_off, atom_off, src, dst), packed, atoms = O.moe_dispatch(x, ids, e)
    ka = k // 64
    assert atoms.shape[0] == int(atom_off[-1]) * ka * 512
    for g in range(e):
        r0, r1 = int(row_off[g]), int(row_off[g + 1])
        rows = x[src[r0:r1]]
        p_ref, sf_ref = O.quantize_nvfp4(rows)
        assert np.array_equal(packed[r0:r1], p_ref)
        blk = atoms[int(atom_off[g]) * ka * 512:int(atom_off[g + 1]) * ka * 512]
        # the expert's atoms are to_blocked of its scales (zero padding)
        assert np.array_equal(blk, O.to_blocked(sf_ref))


def test_oracle_combine_loop():
    rng = np.random.default_rng(6)
    t, topk, n = 20, 2, 24
    c = rng.standard_normal((t * topk, n)).astype(np.float16)
    dst = rng.permutation(t * topk)
    dst[3] = -1
    w = rng.random((t, topk)).astype(np.float32)
    out = O.moe_combine(c, dst, w, t, topk)
    for ti in range(t):
        for col in range(n):
            acc = np.float32(0)
            for j in range(topk):
                r = dst[ti * topk + j]
                if r >= 0:
                    acc = np.float32(acc + np.float32(w[ti, j] * np.float32(c[r, col])))
            assert out[ti, col] == acc


# ----------------------------------------------------------------------------
# GPU: the CUDA path against the oracle
# ----------------------------------------------------------------------------
def _gpu_dispatch(x, ids, e):
    from nvfp4_b200 import moe
    d = moe.dispatch(x.cuda(), ids.cuda(), e)
    torch.cuda.synchronize()
    return d


def _check_dispatch(d, x, ids, e):
    topk = ids.shape[1] if ids.dim() == 2 else 1
    (counts, row_off, atom_off, src, dst), packed, atoms = O.moe_dispatch(
        x.numpy(), ids.numpy().reshape(x.shape[0], topk), e)
    rows = int(row_off[-1])
    assert d.counts.cpu().tolist() == counts.tolist()
    assert d.row_offsets.cpu().tolist() == row_off.tolist()
    assert d.atom_offsets.cpu().tolist() == atom_off.tolist()
    assert d.src.cpu()[:rows].tolist() == src.tolist()
    assert d.dst.cpu().tolist() == dst.tolist()
    assert np.array_equal(d.packed.cpu().numpy()[:rows], packed)
    assert np.array_equal(d.sf.cpu().numpy()[:atoms.shape[0]], atoms)


@pytest.mark.gpu
@pytest.mark.parametrize("t,topk,e,k,lo,hi", [
    (1000, 1, 8, 256, 0, 8),            # plain top-1
    (333, 2, 5, 128, -1, 7),            # top-2 with dropped ids on both sides
    (700, 1, 1, 64, 0, 1),              # one expert: several 128-row blocks
    (64, 4, 1024, 192, 0, 1024),        # many experts, most empty
    (3000, 2, 64, 512, 0, 64),          # several chunks of 1024 pairs
    (5, 1, 3, 7168, 0, 3),              # configuration 4's K, tiny token count
])
def test_dispatch_matches_oracle(t, topk, e, k, lo, hi):
    g = torch.Generator().manual_seed(t + e)
    x = torch.randn(t, k, generator=g)
    ids = torch.randint(lo, hi, (t, topk), generator=g, dtype=torch.int32)
    _check_dispatch(_gpu_dispatch(x, ids, e), x, ids, e)


@pytest.mark.gpu
def test_dispatch_no_tokens_and_all_dropped():
    from nvfp4_b200 import moe
    x = torch.zeros(0, 64, device="cuda")
    d = moe.dispatch(x, torch.zeros(0, dtype=torch.int32, device="cuda"), 4)
    assert d.counts.cpu().tolist() == [0] * 4 and d.row_offsets.cpu().tolist() == [0] * 5
    x = torch.randn(40, 64)
    ids = torch.full((40, 1), 9, dtype=torch.int32)
    d = _gpu_dispatch(x, ids, 4)
    assert d.counts.cpu().tolist() == [0] * 4 and d.dst.cpu().tolist() == [-1] * 40


@pytest.mark.gpu
def test_dispatch_reuses_out_and_is_deterministic():
    from nvfp4_b200 import moe
    g = torch.Generator().manual_seed(9)
    x = torch.randn(2500, 128, generator=g).cuda()
    ids = torch.randint(0, 16, (2500, 2), generator=g, dtype=torch.int32).cuda()
    d = moe.dispatch(x, ids, 16)
    first = (d.src.clone(), d.packed.clone(), d.sf.clone())
    d2 = moe.dispatch(x, ids, 16, out=d)
    assert d2 is d
    assert all(torch.equal(a, b) for a, b in zip(first, (d.src, d.packed, d.sf)))


@pytest.mark.gpu
def test_dispatch_config4_routing_full_size_properties():
    """Configuration 4's routing (32768 tokens, Zipf over 64 experts) at its
    K = 7168: counts equal the configuration's M_g, src / dst are inverse
    permutations in stable order, and sampled rows of every expert are
    quantised bit-exactly."""
    from nvfp4_b200 import inputs as I
    from nvfp4_b200 import moe
    ids = I.config4_expert_ids()
    g = torch.Generator().manual_seed(4)
    x = torch.randn(32768, 7168, generator=g)
    d = moe.dispatch(x.cuda(), ids.cuda(), 64)
    counts = d.counts.cpu()
    assert counts.tolist() == I.config4_m_sizes()
    src, dst = d.src.cpu().long(), d.dst.cpu().long()
    assert torch.equal(dst[src], torch.arange(32768))
    row_off = d.row_offsets.cpu().tolist()
    eid = ids.long()[src]
    assert torch.equal(eid, torch.repeat_interleave(torch.arange(64), counts.long()))
    for e in range(64):                                   # stable: ascending tokens per expert
        seg = src[row_off[e]:row_off[e + 1]]
        assert bool((seg[1:] > seg[:-1]).all())
    ka = 7168 // 64
    packed, sf = d.packed, d.sf
    atom_off = d.atom_offsets.cpu().tolist()
    for e in range(0, 64, 7):
        m = counts[e].item()
        if m == 0:
            continue
        take = sorted({0, m - 1, m // 2})
        rows = x[src[row_off[e]:row_off[e + 1]][take]].numpy()
        p_ref, sf_ref = O.quantize_nvfp4(rows)
        got = packed[[row_off[e] + i for i in take]].cpu().numpy()
        assert np.array_equal(got, p_ref)
        atoms = sf[atom_off[e] * ka * 512:atom_off[e + 1] * ka * 512].cpu().numpy()
        plain = O.unpermute_sf(atoms.reshape(1, -1, ka, 32, 4, 4), m, 7168 // 16)[:, :, 0]
        assert np.array_equal(plain[take], sf_ref)


@pytest.mark.gpu
@pytest.mark.parametrize("t,topk,n,weighted", [(100, 1, 256, False), (77, 2, 200, True),
                                                (33, 3, 1000, True), (5, 2, 8, True)])
def test_combine_matches_oracle(t, topk, n, weighted):
    from nvfp4_b200 import moe
    g = torch.Generator().manual_seed(t * n)
    ids = torch.randint(-1, 6, (t, topk), generator=g, dtype=torch.int32)
    d = _gpu_dispatch(torch.randn(t, 64, generator=g), ids, 6)
    rows = t * topk
    c = torch.randn(rows, n, generator=g).half()
    w = torch.rand(t, topk, generator=g) if weighted else None
    out = moe.combine(c.cuda(), d, w.cuda() if w is not None else None)
    ref = O.moe_combine(c.numpy(), d.dst.cpu().numpy(), None if w is None else w.numpy(), t, topk)
    assert np.array_equal(out.cpu().numpy(), ref)


@pytest.mark.gpu
def test_moe_layer_dispatch_grouped_combine():
    """Tokens -> dispatch -> grouped GEMM (per-expert NVFP4 weights) ->
    combine, against the oracle's route + quantise + per-expert GEMM + combine."""
    from nvfp4_b200 import group_gemm as G
    from nvfp4_b200 import moe
    from nvfp4_b200.formats import quantize_nvfp4, swizzle_sf
    g = torch.Generator().manual_seed(11)
    t, topk, e, k, n = 600, 2, 6, 512, 256
    x = torch.randn(t, k, generator=g)
    ids = torch.randint(0, e, (t, topk), generator=g, dtype=torch.int32)
    ws = [torch.randn(n, k, generator=g) for _ in range(e)]
    wq = []
    for w in ws:
        packed, sf = quantize_nvfp4(w)
        wq.append((packed.view(torch.float4_e2m1fn_x2).unsqueeze(-1).cuda(),
                   swizzle_sf(sf.unsqueeze(-1)).cuda(), packed, sf))
    d = moe.dispatch(x.cuda(), ids.cuda(), e)
    c_all = torch.zeros(t * topk, n, dtype=torch.float16, device="cuda")
    data, which = moe.grouped_inputs(d, [(a, s) for a, s, _, _ in wq], c_all)
    G.custom_kernel(data)
    weights = torch.rand(t, topk, generator=g)
    out = moe.combine(c_all, d, weights.cuda()).cpu().numpy()
    # oracle: route + quantise the tokens, per-expert fp16 GEMM, combine
    (counts, row_off, _, src, dst), a_packed, _ = O.moe_dispatch(x.numpy(), ids.numpy(), e)
    _, a_sf = O.quantize_nvfp4(x.numpy()[src // topk])
    c_ref = np.zeros((t * topk, n), np.float16)
    for ex in range(e):
        r0, r1 = int(row_off[ex]), int(row_off[ex + 1])
        if r1 > r0:
            c_ref[r0:r1] = O.ref_group(a_packed[r0:r1], wq[ex][2].numpy(), a_sf[r0:r1],
                                       wq[ex][3].numpy())
    nbad, idx = O.allclose_report(c_all.cpu().numpy(), c_ref, 1e-2, 1e-2)
    assert nbad == 0, idx
    ref = O.moe_combine(c_ref, dst, weights.numpy(), t, topk)
    nbad, idx = O.allclose_report(out, ref, 1e-2, 1e-2)
    assert nbad == 0, idx
    assert which == [ex for ex in range(e) if counts[ex] > 0]


def _moe_weights(e, n, k, seed):
    from nvfp4_b200.formats import quantize_nvfp4, swizzle_sf
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(e):
        packed, sf = quantize_nvfp4(torch.randn(n, k, generator=g))
        out.append((packed.view(torch.float4_e2m1fn_x2).unsqueeze(-1).cuda(),
                    swizzle_sf(sf.unsqueeze(-1)).cuda()))
    return out


@pytest.mark.gpu
@pytest.mark.parametrize("t,topk,e,n,k,lo", [(600, 2, 6, 256, 512, 0), (333, 1, 5, 384, 256, -1),
                                             (1000, 1, 3, 128, 512, 0), (50, 2, 130, 256, 256, 0)])
def test_moe_grouped_gemm_matches_host_table_path(t, topk, e, n, k, lo):
    """The device-routed grouped GEMM (sizes read on the device) gives exactly
    the grouped GEMM of the host-table path on the same dispatch."""
    from nvfp4_b200 import group_gemm as G
    from nvfp4_b200 import moe
    g = torch.Generator().manual_seed(t + e)
    x = torch.randn(t, k, generator=g).cuda()
    ids = torch.randint(lo, e, (t, topk), generator=g, dtype=torch.int32).cuda()
    w = _moe_weights(e, n, k, seed=e)
    d = moe.dispatch(x, ids, e)
    c_dev = torch.full((t * topk, n), float("nan"), dtype=torch.float16, device="cuda")
    moe.grouped_gemm(d, moe.ExpertWeights(w), c_dev)
    c_host = torch.full((t * topk, n), float("nan"), dtype=torch.float16, device="cuda")
    data, _ = moe.grouped_inputs(d, w, c_host)
    G.custom_kernel(data)
    rows = int(d.row_offsets[-1].item())
    assert torch.equal(c_dev[:rows], c_host[:rows])
    assert _lib_status() == 0


def _lib_status():
    from nvfp4_b200 import _lib
    return _lib.device_status()


@pytest.mark.gpu
def test_moe_layer_captured_in_a_cuda_graph():
    """dispatch -> device-routed grouped GEMM -> combine, captured once in a
    CUDA graph (no host synchronisation inside) and replayed on new tokens
    and new routing: equal to the eager layer on the same inputs."""
    from nvfp4_b200 import moe
    t, topk, e, n, k = 512, 2, 8, 256, 512
    g = torch.Generator().manual_seed(21)
    w = moe.ExpertWeights(_moe_weights(e, n, k, seed=3))
    x = torch.randn(t, k, generator=g).cuda()
    ids = torch.randint(0, e, (t, topk), generator=g, dtype=torch.int32).cuda()
    rw = torch.rand(t, topk, generator=g).cuda()
    d = moe.dispatch(x, ids, e)                            # buffers for the captured calls
    c_all = torch.zeros(t * topk, n, dtype=torch.float16, device="cuda")
    out = torch.zeros(t, n, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        moe.dispatch(x, ids, e, out=d)
        moe.grouped_gemm(d, w, c_all)
        moe.combine(c_all, d, rw, out=out)
        torch.cuda.synchronize()
        with torch.cuda.graph(graph, stream=s):
            moe.dispatch(x, ids, e, out=d)
            moe.grouped_gemm(d, w, c_all)
            moe.combine(c_all, d, rw, out=out)
    for seed in (5, 6):
        gg = torch.Generator().manual_seed(seed)
        x.copy_(torch.randn(t, k, generator=gg))
        ids.copy_(torch.randint(0, e, (t, topk), generator=gg, dtype=torch.int32))
        rw.copy_(torch.rand(t, topk, generator=gg))
        graph.replay()
        torch.cuda.synchronize()
        got = out.clone()
        d2 = moe.dispatch(x, ids, e)
        c2 = torch.zeros_like(c_all)
        moe.grouped_gemm(d2, w, c2)
        ref = moe.combine(c2, d2, rw)
        torch.cuda.synchronize()
        assert torch.equal(got, ref)
    del graph
