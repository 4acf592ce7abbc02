"""Batched decode over the union of up to 8 tokens' active groups
(ls_b200_batch_mlp): with the per-token mask each token's output equals the
one-token oracle over its own groups; without it, the oracle over the whole
union; within the output tolerance of the one-token path (2e-3 of max|y|).
Partial batches, the fp32 output, the residual and determinism (two calls,
identical bits) are checked too; H 1024 and 8192 (config 5's geometry)."""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _run(lib, H, G, L, union_rows, x, mask, tokens, residual=None):
    import torch
    from leanstream_b200 import _native as N

    dev = "cuda"
    U = len(union_rows)
    cache = torch.from_numpy(L.packed).to(dev)
    scales = torch.from_numpy(L.scales.reshape(-1).view(np.int16)).to(dev)
    desc = torch.from_numpy(np.ascontiguousarray(union_rows, dtype=np.uint32).reshape(-1).view(np.int32)).to(dev)
    xt = torch.from_numpy(np.ascontiguousarray(x).view(np.int16)).to(dev)
    y = torch.zeros(tokens, H, dtype=torch.int16, device=dev)
    y32 = torch.zeros(tokens, H, dtype=torch.float32, device=dev)
    mk = torch.from_numpy(np.ascontiguousarray(mask, dtype=np.uint8)).to(dev) if mask is not None else None
    res = torch.from_numpy(np.ascontiguousarray(residual).view(np.int16)).to(dev) if residual is not None else None
    hid = torch.zeros(tokens, H, dtype=torch.int16, device=dev) if residual is not None else None
    nbytes = int(lib.ls_b200_batch_scratch_bytes(H, G, U))
    scratch = torch.full((nbytes,), 0xFF, dtype=torch.uint8, device=dev)  # stale bytes: must not leak in
    a = N.BatchArgs(H, G, U, tokens, xt.data_ptr(), y.data_ptr(), y32.data_ptr(),
                    res.data_ptr() if res is not None else None, hid.data_ptr() if hid is not None else None,
                    cache.data_ptr(), None, scales.data_ptr(), desc.data_ptr(),
                    mk.data_ptr() if mk is not None else None, scratch.data_ptr(), nbytes)
    assert lib.ls_b200_batch_mlp(C.byref(a), torch.cuda.current_stream().cuda_stream) == 0
    torch.cuda.synchronize()
    out = (y.cpu().numpy().view(np.float16), y32.cpu().numpy())
    return out + ((hid.cpu().numpy().view(np.float16),) if hid is not None else ())


@pytest.mark.parametrize("H,n_groups", [(1024, 32), (8192, 20)])
def test_batch_matches_one_token_oracle(native_lib, cuda_device, H, n_groups):
    from leanstream_b200.synthetic import descriptors, make_layer
    from oracle import oracle as O

    G, B = 64, 8
    L = make_layer(17, H, n_groups, G)
    rng = np.random.default_rng(3)
    sets = [np.sort(rng.permutation(n_groups)[: rng.integers(3, n_groups // 2)]) for _ in range(B)]
    union = np.unique(np.concatenate(sets))
    rows = descriptors(union)
    x = (rng.standard_normal((B, H)) * 0.5).astype(np.float16)
    mask = np.array([[u in set(s.tolist()) for u in union] for s in sets], np.uint8)
    y, y32 = _run(native_lib, H, G, L, rows, x, mask, B)
    y_again, _ = _run(native_lib, H, G, L, rows, x, mask, B)
    assert np.array_equal(y.view(np.uint16), y_again.view(np.uint16)), "deterministic"
    for b in range(B):
        ref, _, _ = O.mlp(H, G, x[b], L.packed, L.scales, descriptors(sets[b]))
        ref = ref.astype(np.float32)
        assert np.abs(y[b].astype(np.float32) - ref).max() <= TOL * np.abs(ref).max(), b
        assert np.array_equal(y[b], y32[b].astype(np.float16))
    # no mask: every token over the whole union
    yu, _ = _run(native_lib, H, G, L, rows, x, None, B)
    for b in (0, B - 1):
        ref, _, _ = O.mlp(H, G, x[b], L.packed, L.scales, rows)
        ref = ref.astype(np.float32)
        assert np.abs(yu[b].astype(np.float32) - ref).max() <= TOL * np.abs(ref).max(), b


def test_partial_batch_with_residual(native_lib, cuda_device):
    from leanstream_b200.synthetic import descriptors, make_layer
    from oracle import oracle as O

    H, G, n_groups, B = 1024, 40, 9, 3  # G not a multiple of 16: neurons past the union's end
    L = make_layer(23, H, n_groups, G)
    rng = np.random.default_rng(8)
    union = np.array([0, 2, 3, 7, 8])
    rows = descriptors(union)
    x = (rng.standard_normal((B, H)) * 0.5).astype(np.float16)
    resid = rng.standard_normal((B, H)).astype(np.float16)
    y, y32, hid = _run(native_lib, H, G, L, rows, x, None, B, residual=resid)
    for b in range(B):
        ref, _, _ = O.mlp(H, G, x[b], L.packed, L.scales, rows)
        ref = ref.astype(np.float32)
        assert np.abs(y[b].astype(np.float32) - ref).max() <= TOL * np.abs(ref).max()
        assert np.array_equal(hid[b].view(np.uint16), O.residual(resid[b], y[b]).view(np.uint16))


@pytest.mark.parametrize("H", [1024, 8192])
def test_batch_norm_chains_layers(native_lib, cuda_device, H):
    """LS_B200_NORM_INPUT with residual and hidden_out: three chained batch
    layers (x_{l+1} = hidden_out of layer l), each token masked to its own
    groups, equal per token the one-token oracle chain
    x_{l+1} = fp16(x_l + MLP(RMSNorm_HF(x_l))) within the output tolerance."""
    import torch
    from leanstream_b200.batch import BatchMLP, union_plan
    from leanstream_b200.synthetic import descriptors, make_layer
    from oracle import oracle as O

    G, n_groups, B, layers = 64, 24, 8, 3
    Ls = [make_layer(60 + l, H, n_groups, G) for l in range(layers)]
    rng = np.random.default_rng(9)
    x0 = (rng.standard_normal((B, H)) * 3.0).astype(np.float16)  # un-normalised: the norm matters
    mlp = BatchMLP(H, G, n_groups, device="cuda")
    xs = [torch.from_numpy(x0.view(np.int16)).cuda().view(torch.float16)]
    y = torch.zeros(B, H, dtype=torch.float16, device="cuda")
    plans = []
    for l in range(layers):
        sets = [np.sort(rng.permutation(n_groups)[: rng.integers(3, 9)]) for _ in range(B)]
        union, rows, mask = union_plan(sets)
        plans.append((sets, union))
        desc = torch.from_numpy(np.ascontiguousarray(rows.reshape(-1).view(np.int32))).cuda()
        mk = torch.from_numpy(np.ascontiguousarray(mask)).cuda()
        cache = torch.from_numpy(Ls[l].packed).cuda()
        scales = torch.from_numpy(Ls[l].scales.reshape(-1).view(np.int16)).cuda().view(torch.float16)
        xs.append(torch.zeros(B, H, dtype=torch.float16, device="cuda"))
        mlp.run(x=xs[l], output=y, cache=cache, scales=scales, union_descs=desc, union_count=len(union),
                tokens=B, mask=mk, residual=xs[l], hidden_out=xs[l + 1], norm_input=True, rms_eps=1e-5)
        torch.cuda.synchronize()
    got = [t.cpu().numpy() for t in xs]
    for b in range(B):
        for l in range(layers):
            x_l = got[l][b]
            assert np.isfinite(x_l.astype(np.float32)).all()
            xin = O.rmsnorm(x_l, None, 1e-5)
            y_ref, _, _ = O.mlp(H, G, xin, Ls[l].packed, Ls[l].scales, descriptors(plans[l][0][b]))
            ref = O.residual(x_l, y_ref).astype(np.float32)
            out = got[l + 1][b].astype(np.float32)
            assert np.abs(out - ref).max() <= TOL * np.abs(ref).max() + 1e-3, (b, l, np.abs(out - ref).max())


@pytest.mark.parametrize("H,n_groups", [(1024, 40), (8192, 24)])
def test_tcgen05_matches_warp_mma(native_lib, cuda_device, H, n_groups):
    """The default tensor-core kernels (tcgen05.mma, accumulator in tensor
    memory) and the legacy warp-level MMA kernels run the same arithmetic
    (w = fp16(q * s), fp32 sums) in different summation orders: their
    outputs agree within the output tolerance, both equal the masked
    one-token oracle, and the tcgen05 error word stays clear."""
    import torch
    from leanstream_b200.batch import BatchMLP, union_plan
    from leanstream_b200.synthetic import descriptors, make_layer
    from oracle import oracle as O

    G, B = 64, 8
    L = make_layer(23, H, n_groups, G)
    rng = np.random.default_rng(5)
    sets = [np.sort(rng.permutation(n_groups)[: rng.integers(4, n_groups // 2)]) for _ in range(B)]
    union, rows, mask = union_plan(sets)
    x = (rng.standard_normal((B, H)) * 0.5).astype(np.float16)
    mlp = BatchMLP(H, G, n_groups, device="cuda")
    cache = torch.from_numpy(L.packed).cuda()
    scales = torch.from_numpy(L.scales.reshape(-1).view(np.int16)).cuda().view(torch.float16)
    desc = torch.from_numpy(np.ascontiguousarray(rows.reshape(-1).view(np.int32))).cuda()
    mk = torch.from_numpy(np.ascontiguousarray(mask)).cuda()
    xt = torch.from_numpy(x.view(np.int16)).cuda().view(torch.float16)
    outs = {}
    for legacy in (False, True):
        y = torch.zeros(B, H, dtype=torch.float16, device="cuda")
        y32 = torch.zeros(B, H, dtype=torch.float32, device="cuda")
        mlp.run(x=xt, output=y, output_f32=y32, cache=cache, scales=scales, union_descs=desc,
                union_count=len(union), tokens=B, mask=mk, mma_sync=legacy)
        torch.cuda.synchronize()
        outs[legacy] = (y.cpu().numpy().astype(np.float32), y32.cpu().numpy())
    assert mlp.error() == 0
    tc, mm = outs[False][1], outs[True][1]
    assert np.isfinite(tc).all()
    assert np.abs(tc - mm).max() <= TOL * np.abs(mm).max(), np.abs(tc - mm).max()
    for b in range(B):
        y_ref, _, _ = O.mlp(H, G, x[b], L.packed, L.scales, descriptors(sets[b]))
        ref = y_ref.astype(np.float32)
        assert np.abs(outs[False][0][b] - ref).max() <= TOL * np.abs(ref).max(), b


def test_tcgen05_bounded_waits_report_and_recover(native_lib, cuda_device):
    """Failure detection without a fault: with a wait bound shorter than the
    work (timeout_ns = 1) the tensor-core kernels' bounded waits give up, the
    call sets bit 0 of the error word and ends (each kernel waits, within a
    further second, for its own copies and MMAs in flight, and frees its
    tensor memory); the next call on the same stream and scratch, with the
    default bound, reports no error and matches the oracle."""
    import torch
    from leanstream_b200.batch import BatchMLP, union_plan
    from leanstream_b200.synthetic import descriptors, make_layer
    from oracle import oracle as O

    H, G, n_groups, B = 1024, 64, 32, 4
    L = make_layer(31, H, n_groups, G)
    rng = np.random.default_rng(9)
    sets = [np.sort(rng.permutation(n_groups)[: rng.integers(6, 14)]) for _ in range(B)]
    union, rows, mask = union_plan(sets)
    x = (rng.standard_normal((B, H)) * 0.5).astype(np.float16)
    mlp = BatchMLP(H, G, n_groups, device="cuda")
    kw = dict(x=torch.from_numpy(x.view(np.int16)).cuda().view(torch.float16),
              cache=torch.from_numpy(L.packed).cuda(),
              scales=torch.from_numpy(L.scales.reshape(-1).view(np.int16)).cuda().view(torch.float16),
              union_descs=torch.from_numpy(np.ascontiguousarray(rows.reshape(-1).view(np.int32))).cuda(),
              union_count=len(union), tokens=B, mask=torch.from_numpy(np.ascontiguousarray(mask)).cuda())
    y = torch.zeros(B, H, dtype=torch.float16, device="cuda")
    mlp.run(output=y, timeout_ns=1, **kw)
    torch.cuda.synchronize()
    assert mlp.error() & 1
    mlp.clear_error()
    y.zero_()
    mlp.run(output=y, **kw)
    torch.cuda.synchronize()
    assert mlp.error() == 0
    got = y.cpu().numpy().astype(np.float32)
    for b in range(B):
        y_ref, _, _ = O.mlp(H, G, x[b], L.packed, L.scales, descriptors(sets[b]))
        ref = y_ref.astype(np.float32)
        assert np.abs(got[b] - ref).max() <= TOL * np.abs(ref).max(), b


def test_tcgen05_edge_geometry_staging(native_lib, cuda_device):
    """The tensor-core kernels' edge paths: a group size that is neither a
    power of two nor a multiple of the 64-neuron tile (G 48: partial gate/up
    tiles, partial 128-neuron down stages, the producer's division path),
    some groups read from the staging buffer (kind 1), cache slots permuted,
    5 tokens at H 2048. Each token matches the oracle over its own set, and
    the warp-MMA kernels agree."""
    import torch
    from leanstream_b200.batch import BatchMLP, union_plan
    from leanstream_b200.synthetic import descriptors, make_layer
    from oracle import oracle as O

    H, G, n_groups, B = 2048, 48, 22, 5
    L = make_layer(77, H, n_groups, G)
    rng = np.random.default_rng(13)
    sets = [np.sort(rng.permutation(n_groups)[: rng.integers(5, 12)]) for _ in range(B)]
    # logical group g sits in cache slot perm[g]
    perm = rng.permutation(n_groups)
    gbytes = G * 3 * H // 2
    packed = L.packed.reshape(n_groups, gbytes)
    cache_np = np.zeros_like(packed)
    cache_np[perm] = packed
    union_all = np.unique(np.concatenate(sets))
    staged = {int(g): i for i, g in enumerate(union_all[::3])}  # every third union group from staging
    staging_np = np.zeros((len(staged), gbytes), np.uint8)
    for g, slot in staged.items():
        staging_np[slot] = packed[g]
    union, rows, mask = union_plan(sets, cache_slots=perm, physical=np.arange(n_groups), staging=staged)
    x = (rng.standard_normal((B, H)) * 0.5).astype(np.float16)
    mlp = BatchMLP(H, G, n_groups, device="cuda")
    kw = dict(x=torch.from_numpy(x.view(np.int16)).cuda().view(torch.float16),
              cache=torch.from_numpy(cache_np.reshape(-1)).cuda(),
              staging=torch.from_numpy(staging_np.reshape(-1)).cuda(),
              scales=torch.from_numpy(L.scales.reshape(-1).view(np.int16)).cuda().view(torch.float16),
              union_descs=torch.from_numpy(np.ascontiguousarray(rows.reshape(-1).view(np.int32))).cuda(),
              union_count=len(union), tokens=B, mask=torch.from_numpy(np.ascontiguousarray(mask)).cuda())
    outs = {}
    for legacy in (False, True):
        y32 = torch.zeros(B, H, dtype=torch.float32, device="cuda")
        y = torch.zeros(B, H, dtype=torch.float16, device="cuda")
        mlp.run(output=y, output_f32=y32, mma_sync=legacy, **kw)
        torch.cuda.synchronize()
        outs[legacy] = (y.cpu().numpy().astype(np.float32), y32.cpu().numpy())
    assert mlp.error() == 0
    tc, mm = outs[False][1], outs[True][1]
    assert np.isfinite(tc).all()
    assert np.abs(tc - mm).max() <= TOL * np.abs(mm).max(), np.abs(tc - mm).max()
    for b in range(B):
        y_ref, _, _ = O.mlp(H, G, x[b], L.packed, L.scales, descriptors(sets[b]))
        ref = y_ref.astype(np.float32)
        assert np.abs(outs[False][0][b] - ref).max() <= TOL * np.abs(ref).max(), b
