"""Device-side failure detection without a fault: a bounded pipeline wait that can never
complete expires, the kernel records its site code and returns, the host reads
FKC_ETIMEOUT, and the context keeps working."""

from __future__ import annotations

import time

import pytest
import torch

from _data import iid, subset_init

pytestmark = pytest.mark.gpu


def test_expired_wait_is_reported_and_context_survives(cuda_device):
    from flash_kmeans_cuda import _lib, euclid_assign

    L = _lib.lib
    st = torch.cuda.current_stream().cuda_stream
    assert L.fkc_device_status() == 0
    t0 = time.perf_counter()
    assert L.fkc_selftest_wait_timeout(50_000, st) == 0  # 50 ms deadline
    status = L.fkc_device_status()  # synchronises
    elapsed = time.perf_counter() - t0
    assert status == -4, _lib.last_error()  # FKC_ETIMEOUT
    assert "site code 199" in _lib.last_error()
    assert 0.04 <= elapsed < 5.0
    assert L.fkc_device_status() == 0  # the record was cleared
    # the context is usable: a normal assignment runs and is right
    x = iid(1, 4096, 64, seed=3).cuda()
    c = subset_init(x.cpu(), 32, seed=4).cuda()
    ids = euclid_assign(x, c, (x.float() ** 2).sum(-1))
    torch.cuda.synchronize()
    d = torch.cdist(x[0].float(), c[0].float())
    assert (ids[0].long() == d.argmin(dim=1)).float().mean().item() > 0.999
    assert L.fkc_device_status() == 0


def test_selftest_rejects_bad_timeout(cuda_device):
    from flash_kmeans_cuda import _lib

    assert _lib.lib.fkc_selftest_wait_timeout(0, None) == -1
    assert "timeout_us" in _lib.last_error()
