"""Update and finalize parity on the GPU, through the C-ABI, against the oracle.

Counts are compared exactly; fp32 sums to the float64 oracle within 1e-5
relative to the row's absolute sum (fp32 accumulation); finalized centroids
within 1e-3 relative. Covers the reference's C++ smoke checks
(tests/cpp/smoke.cpp:58-95: sorted == indexed sums/counts, finalize ==
where(count>0, sums/count, old)) at D in {1, 7, 16, 31, 32, 64, 128, 257}.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle.lloyd as orc
from _data import iid, mixture, to_np

pytestmark = pytest.mark.gpu


def _labels(B, N, K, seed, zipf=0.0):
    g = torch.Generator().manual_seed(seed)
    if zipf > 0:
        p = torch.arange(1, K + 1, dtype=torch.float64) ** (-zipf)
        lab = torch.multinomial(p / p.sum(), B * N, replacement=True, generator=g)
        return lab.view(B, N).to(torch.int32)
    return torch.randint(0, K, (B, N), generator=g, dtype=torch.int32)


def _check_sums(sums, counts, x_np, ids_np, K):
    ref_s, ref_c = orc.update(x_np, ids_np, K)
    assert np.array_equal(counts, ref_c), "counts differ"
    scale = orc.update(np.abs(x_np), ids_np, K)[0] + 1e-6
    err = np.abs(sums - ref_s) / scale
    assert err.max() < 1e-5, f"sums rel err {err.max():.3g}"


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("B,N,K,D,zipf", [
    (1, 4096, 64, 128, 0.0),
    (1, 65536, 2048, 128, 1.1),
    (2, 10000, 300, 64, 0.0),
    (1, 5000, 17, 96, 1.1),
    (3, 3000, 1000, 32, 0.0),
    (1, 2000, 50, 7, 0.0),
    (1, 2000, 50, 257, 0.0),
    (1, 1, 1, 128, 0.0),
])
def test_update_counting_sort(cuda_device, dtype, B, N, K, D, zipf):
    from flash_kmeans_cuda import centroid_update_sorted

    x = iid(B, N, D, seed=N + D, dtype=dtype)
    ids = _labels(B, N, K, seed=K, zipf=zipf)
    sums = torch.full((B, K, D), 123.0, device="cuda")  # must be overwritten
    counts = torch.full((B, K), 7, dtype=torch.int32, device="cuda")
    s, c = centroid_update_sorted(x.cuda(), ids.cuda(), K, sums_out=sums, counts_out=counts)
    torch.cuda.synchronize()
    _check_sums(s.cpu().numpy(), c.cpu().numpy(), to_np(x), ids.numpy(), K)


@pytest.mark.parametrize("N,K,zipf", [
    (700_000, 4096, 0.0),      # 2048-row scatter chunks
    (1_300_000, 16384, 1.1),   # 4096-row chunks, the largest K with shared-memory ranks
    (1_300_000, 16385, 1.1),   # the per-row atomic scatter just above it
])
def test_counting_sort_large_chunks(cuda_device, N, K, zipf):
    """Scatter chunk sizes that only large N selects, with a dominant Zipf cluster."""
    from flash_kmeans_cuda import centroid_update_sorted

    x = iid(1, N, 4, seed=N, dtype="float32")
    ids = _labels(1, N, K, seed=K, zipf=zipf)
    s, c = centroid_update_sorted(x.cuda(), ids.cuda(), K)
    torch.cuda.synchronize()
    _check_sums(s.cpu().numpy(), c.cpu().numpy(), to_np(x), ids.numpy(), K)


@pytest.mark.parametrize("D", [1, 7, 16, 31, 32, 64, 128, 257])
def test_sorted_and_indexed_match(cuda_device, D):
    """Reference _C semantics: accumulate into pre-zeroed buffers from sorted runs."""
    from flash_kmeans_cuda import _C

    B, N, K = 1, 512, 16
    x = torch.randn(B, N, D, device="cuda")
    ids = torch.randint(0, K, (B, N), device="cuda", dtype=torch.int32)
    sorted_ids, perm = torch.sort(ids, dim=1)
    sorted_ids = sorted_ids.contiguous()
    perm32 = perm.to(torch.int32).contiguous()
    x_sorted = torch.gather(x, 1, perm.unsqueeze(-1).expand(-1, -1, D)).contiguous()
    s1 = torch.zeros(B, K, D, device="cuda")
    c1 = torch.zeros(B, K, dtype=torch.int32, device="cuda")
    _C.centroid_update_sorted(x_sorted, sorted_ids, s1, c1)
    s2 = torch.zeros_like(s1)
    c2 = torch.zeros_like(c1)
    _C.centroid_update_sorted_indexed(x, perm32, sorted_ids, s2, c2)
    torch.cuda.synchronize()
    assert torch.equal(c1, c2)
    assert torch.allclose(s1, s2, rtol=1e-4, atol=1e-4)
    _check_sums(s1.cpu().numpy(), c1.cpu().numpy(), x.cpu().numpy(), ids.cpu().numpy(), K)
    # accumulation semantics: a second call doubles
    _C.centroid_update_sorted(x_sorted, sorted_ids, s1, c1)
    torch.cuda.synchronize()
    assert torch.equal(c1, 2 * c2)


@pytest.mark.parametrize("dtype", ["float16", "bfloat16", "float32"])
@pytest.mark.parametrize("D", [1, 7, 64, 128, 257])
def test_finalize(cuda_device, dtype, D):
    from flash_kmeans_cuda import centroid_finalize
    from _data import TORCH_DTYPES

    B, K = 2, 33
    g = torch.Generator().manual_seed(D)
    sums = torch.randn(B, K, D, generator=g) * 50
    counts = torch.randint(0, 5, (B, K), generator=g, dtype=torch.int32)
    old = torch.randn(B, K, D, generator=g).to(TORCH_DTYPES[dtype])
    new = centroid_finalize(sums.cuda(), counts.cuda(), old.cuda())
    torch.cuda.synchronize()
    ref = orc.finalize(sums.numpy(), counts.numpy(), to_np(old), dtype)
    got = to_np(new)
    empty = counts.numpy() == 0
    assert np.array_equal(got[empty], to_np(old)[empty]), "empty clusters must keep old"
    rel = np.abs(got - ref) / (np.abs(ref) + 1e-6)
    assert rel.max() < 1e-3
    # in place
    buf = old.cuda().clone()
    centroid_finalize(sums.cuda(), counts.cuda(), buf, out=buf)
    torch.cuda.synchronize()
    assert np.array_equal(to_np(buf), got)


def test_lloyd_step_pieces(cuda_device):
    """fkc_lloyd_local/finalize: ids, fused histogram, sums, c_sq-free next step, shift."""
    from flash_kmeans_cuda.kmeans import LloydState

    x = mixture(1, 30000, 128, 500, seed=3, zipf=1.1).cuda()
    K = 512
    c0 = x[:, :K].contiguous()
    st = LloydState(x, K)
    st.set_centroids(c0)
    st.local(c0)
    new = torch.empty_like(c0)
    st.finalize(c0, new, True)
    torch.cuda.synchronize()
    xn, cn = to_np(x), to_np(c0)
    ref = orc.assign(xn, cn)
    ids = st.ids.cpu().numpy()
    assert not ((ids != ref.ids) & ref.gap_mask()).any()
    _check_sums(st.sums.cpu().numpy(), st.counts.cpu().numpy(), xn, ids, K)
    s_ref, c_ref = orc.update(xn, ids, K)
    fin = orc.finalize(s_ref, c_ref, cn, "float16")
    got = to_np(new)
    assert (np.abs(got - fin) / (np.abs(fin) + 1e-3)).max() < 1e-3
    assert abs(st.shift.item() - orc.shift(got, cn)) < 1e-3 * max(1.0, orc.shift(got, cn))
