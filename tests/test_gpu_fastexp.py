"""The selector's table-driven double exp for non-positive arguments against CUDA's exp (torch's
CUDA float64 exp): at most 2 ulp apart over the selector's whole input range, exact at 0, and
identical below -708 where it defers to CUDA's exp."""
from __future__ import annotations

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def test_exp_nonpos_within_two_ulp_of_cuda_exp():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from diffusorrt_b200 import _lib, build
    build.build()
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(3)
    ln2_32 = float(np.log(2.0) / 32)
    special = torch.tensor([0.0, -0.0, -1e-300, -5e-324, -1e-17, -1e-8, -0.5 * ln2_32, -ln2_32, -708.0, -708.3,
                            -708.4, -709.0, -744.0, -745.2, float("-inf")], dtype=torch.float64, device=dev)
    grid = -torch.arange(0, 708 * 32, dtype=torch.float64, device=dev) * ln2_32  # reduction boundaries
    x = torch.cat([special, -torch.rand(1 << 20, generator=g, device=dev, dtype=torch.float64) * 745.0,
                   -torch.rand(1 << 18, generator=g, device=dev, dtype=torch.float64) * 40.0, grid, grid - 1e-12])
    y = torch.empty_like(x)
    _lib.check(_lib.load().drt_exp_nonpos(x.data_ptr(), y.data_ptr(), x.numel(), torch.cuda.current_stream().cuda_stream))
    ref = torch.exp(x)
    torch.cuda.synchronize()
    xs, ys, rs = x.cpu().numpy(), y.cpu().numpy(), ref.cpu().numpy()
    assert ys[0] == 1.0 and ys[1] == 1.0
    normal = rs >= np.finfo(np.float64).tiny
    ulp = np.spacing(rs[normal])
    err = np.abs(ys[normal] - rs[normal]) / ulp
    assert err.max() <= 2.0, (err.max(), xs[normal][np.argmax(err)])
    sub = ~normal
    assert np.array_equal(ys[sub], rs[sub])
