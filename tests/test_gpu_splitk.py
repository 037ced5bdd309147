"""K-split of the persistent GEMM kernels (ee_gemm.cuh).  With room for partial sums in the
gated workspace (EntropyRouter(k_split=True), ee_gated_workspace_split_bytes), calls with
few tiles for the SMs and long K loops (K >= 8192; 65..128 rows on the single-CTA kernel,
a few hundred rows on the CTA-pair kernel) cut each tile's K loop into ranges run by
different CTAs,
and reduce_partials_kernel adds the ranges' int32 / fp32 partials in range order before
the epilogue.  Checked against the unsplit run of the same routing and against the
reference restatements: INT8 rows bit-identical to both, FP8 / FP16 rows within the
reference tolerance and within the last bits of the unsplit run; buckets of every size,
CTA-pair half tiles, the SwiGLU epilogue, repeated calls on one workspace."""
import pytest
import torch

pytestmark = pytest.mark.gpu

from test_gpu_gated import _ref_fp8, _ref_fp16, _ref_int8, _relf  # noqa: E402


def _inputs(counts, K, N, seed, cuda):
    M = sum(counts)
    g = torch.Generator(device=cuda).manual_seed(seed)
    H = torch.cat([torch.full((c,), v, device=cuda) for c, v in zip(counts, (0.1, 1.0, 3.0))])
    H = H[torch.randperm(M, generator=g, device=cuda)]
    a = torch.randn(M, K, generator=g, device=cuda)
    a = torch.where(torch.rand(M, K, generator=g, device=cuda) < 0.01, a * 20.0, a).half()
    w = (torch.randn(N, K, generator=g, device=cuda) * 0.02).half()
    return H, a, w


def _route(pkg, H, K, k_split, cuda):
    r = pkg.EntropyRouter(0.41, 1.68, k_split=k_split)
    r.reserve(H.shape[0], K, cuda)
    r.route_entropy(H)
    return r


# (INT8, FP8, FP16) rows: the config-3 mixes at 128 and 1024 rows, CTA-pair half tiles
# (buckets of <= 128 rows past a 256-row boundary), single buckets, empty buckets
CASES = [
    ((26, 77, 25), 14336, 4096),
    ((20, 80, 28), 4096, 4096),
    ((30, 20, 15), 8192, 2048),
    ((0, 128, 0), 4096, 1024),
    ((223, 585, 216), 4096, 4096),
    ((243, 556, 225), 14336, 1024),
    ((100, 0, 300), 4096, 2048),
    ((1, 510, 1), 2048, 512),
    ((0, 0, 700), 8192, 768),
]


@pytest.mark.parametrize("counts,K,N", CASES)
def test_split_equals_unsplit_and_reference(pkg, cuda, counts, K, N):
    H, a, w = _inputs(counts, K, N, sum(counts) + K + N, cuda)
    p = pkg.WeightPack(*pkg.quantize_weights_int8(w))
    r0 = _route(pkg, H, K, False, cuda)
    y0 = r0.gated_linear(a, p)
    r1 = _route(pkg, H, K, True, cuda)
    y1 = r1.gated_linear(a, p)
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    assert r1.counts.cpu().tolist() == list(counts)
    route = r1.route_ids
    rows = [torch.nonzero(route == b).flatten() for b in range(3)]
    if rows[0].numel():
        assert torch.equal(y1[rows[0]].view(torch.int16), y0[rows[0]].view(torch.int16))
        assert torch.equal(y1[rows[0]].view(torch.int16), _ref_int8(a[rows[0]], p).view(torch.int16))
    if rows[1].numel():
        assert _relf(y1[rows[1]], _ref_fp8(a[rows[1]], p)) < 1e-2
        assert _relf(y1[rows[1]], y0[rows[1]]) < 1e-3
    if rows[2].numel():
        assert _relf(y1[rows[2]], _ref_fp16(a[rows[2]], p)) < 1e-2
        assert _relf(y1[rows[2]], y0[rows[2]]) < 1e-3


@pytest.mark.parametrize("counts,K,I", [((26, 77, 25), 8192, 1792), ((223, 585, 216), 8192, 1024),
                                        ((0, 300, 0), 14336, 512), ((40, 40, 40), 4096, 512)])
def test_split_swiglu(pkg, cuda, counts, K, I):
    """The SwiGLU epilogue on summed partials: INT8 rows bit-identical to the unsplit
    fused GEMM (exact gate and up accumulators), the other rows within its last bits."""
    H, a, _ = _inputs(counts, K, 8, sum(counts) + I, cuda)
    g = torch.Generator(device=cuda).manual_seed(I)
    gate = pkg.WeightPack(*pkg.quantize_weights_int8((torch.randn(I, K, generator=g, device=cuda) * 0.02).half()))
    up = pkg.WeightPack(*pkg.quantize_weights_int8((torch.randn(I, K, generator=g, device=cuda) * 0.02).half()))
    sp = pkg.SwiGLUPack(gate, up)
    outs = []
    for ks in (False, True):
        r = _route(pkg, H, K, ks, cuda)
        r.pack_rows(a)
        outs.append((r.swiglu_packed(sp), r.route_ids.clone()))
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    (y0, route), (y1, _) = outs
    i8 = torch.nonzero(route == 0).flatten()
    rest = torch.nonzero(route != 0).flatten()
    if i8.numel():
        assert torch.equal(y1[i8].view(torch.int16), y0[i8].view(torch.int16))
    if rest.numel():
        assert _relf(y1[rest], y0[rest]) < 2e-3


def test_split_repeated_calls_one_workspace(pkg, cuda):
    """Three projections per routing, five routings, one workspace (as the Llama block
    runs them): the partial area holds no state between calls."""
    counts, K = (20, 80, 28), 14336
    H, a, _ = _inputs(counts, K, 8, 5, cuda)
    g = torch.Generator(device=cuda).manual_seed(6)
    packs = [pkg.WeightPack(*pkg.quantize_weights_int8((torch.randn(N, K, generator=g, device=cuda) * 0.02).half()))
             for N in (4096, 1024, 2048)]
    r = _route(pkg, H, K, True, cuda)
    first = [r.gated_linear(a, p) for p in packs]
    for _ in range(4):
        r.route_entropy(H)
        again = [r.gated_linear(a, p) for p in packs]
        for x, y in zip(first, again):
            assert torch.equal(x.view(torch.int16), y.view(torch.int16))  # deterministic
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0



@pytest.mark.parametrize("counts,whole_8bit", [((32, 704, 32), True), ((194, 447, 127), False)])
def test_pair_split_between_512_and_768_rows(pkg, cuda, counts, whole_8bit):
    """768 rows x K 14336 on the CTA-pair kernel (forced: the automatic policy takes
    single-CTA tiles there), where the host lets the device plan a K split with up to two
    tiles per pair.  With a small FP16 bucket the FP16 tiles (twice
    the 8-bit K loop) set the makespan and the plan splits them alone: INT8 and FP8 rows
    identical to the unsplit run (their tiles ran whole).  With the bench's routing mix
    the plan splits every bucket (one range length for all).  Either way the split
    rows are not identical to the unsplit run (summed from ranges) but within its last
    bits and the reference tolerance, and INT8 rows equal the reference formula."""
    K, N = 14336, 4096
    H, a, w = _inputs(counts, K, N, 768, cuda)
    p = pkg.WeightPack(*pkg.quantize_weights_int8(w))
    lib = pkg.load_library()
    assert lib.ee_set_gemm_policy(2) == 0
    try:
        y0 = _route(pkg, H, K, False, cuda).gated_linear(a, p)
        r1 = _route(pkg, H, K, True, cuda)
        y1 = r1.gated_linear(a, p)
        torch.cuda.synchronize()
    finally:
        assert lib.ee_set_gemm_policy(0) == 0
    assert pkg._lib.device_check() == 0
    rows = [torch.nonzero(r1.route_ids == b).flatten() for b in range(3)]
    same = [torch.equal(y1[r].view(torch.int16), y0[r].view(torch.int16)) for r in rows]
    assert same[0]
    assert same[1] == whole_8bit
    assert not same[2]
    for b, ref in ((1, _ref_fp8), (2, _ref_fp16)):
        assert _relf(y1[rows[b]], y0[rows[b]]) < 1e-3
        assert _relf(y1[rows[b]], ref(a[rows[b]], p)) < 1e-2
    assert torch.equal(y1[rows[0]].view(torch.int16), _ref_int8(a[rows[0]], p).view(torch.int16))


@pytest.mark.parametrize("counts,whole_8bit", [((194, 447, 127), True), ((120, 300, 200), True),
                                               ((150, 400, 150), False)])
def test_single_cta_split_between_512_and_768_rows(pkg, cuda, counts, whole_8bit):
    """513..768 rows x K 14336 x N 4096: the automatic policy takes single-CTA 128 x 256
    tiles with the K split.  With 128-row tiles the 8-bit tiles fit in one round, so for
    the bench's routing mix at 768 rows (and a larger FP16 share at 620) the plan splits
    the FP16 tiles alone; with a third FP16 tile row it splits every bucket.  Against the
    single-CTA kernel without split room (forced): INT8 rows identical, FP8 rows identical
    when their tiles ran whole on the same kernel, FP16 rows not identical (summed from
    ranges) but within the unsplit run's last bits and the reference tolerance."""
    K, N = 14336, 4096
    H, a, w = _inputs(counts, K, N, sum(counts) + 1, cuda)
    p = pkg.WeightPack(*pkg.quantize_weights_int8(w))
    lib = pkg.load_library()
    assert lib.ee_set_gemm_policy(1) == 0
    try:
        y0 = _route(pkg, H, K, False, cuda).gated_linear(a, p)
    finally:
        assert lib.ee_set_gemm_policy(0) == 0
    r1 = _route(pkg, H, K, True, cuda)
    y1 = r1.gated_linear(a, p)
    torch.cuda.synchronize()
    assert pkg._lib.device_check() == 0
    rows = [torch.nonzero(r1.route_ids == b).flatten() for b in range(3)]
    same = [torch.equal(y1[r].view(torch.int16), y0[r].view(torch.int16)) for r in rows]
    assert same[0]
    assert same[1] == whole_8bit
    assert not same[2]
    for b, ref in ((1, _ref_fp8), (2, _ref_fp16)):
        assert _relf(y1[rows[b]], y0[rows[b]]) < 1e-3
        assert _relf(y1[rows[b]], ref(a[rows[b]], p)) < 1e-2
    assert torch.equal(y1[rows[0]].view(torch.int16), _ref_int8(a[rows[0]], p).view(torch.int16))
