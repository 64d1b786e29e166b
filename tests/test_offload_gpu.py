"""Host-memory pipelined forward+backward (fpscan_b200.offload) against the
device-resident path (the same kernels; few-row device calls may take the
split-row forward, so the comparison is within the normwise tolerance)."""
import pytest
import torch

import fpscan_b200 as fp
from fpscan_b200.offload import scan_fwd_bwd_host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape,block_bytes,depth", [((2, 37, 1024), 8 << 10, 3),
                                                     ((3, 64, 8192), 1 << 20, 2),
                                                     ((1, 5, 65536), 256 << 10, 3),
                                                     ((2, 3, 32), 128 << 20, 3)])
def test_offload_matches_device_path(dtype, shape, block_bytes, depth):
    gen = torch.Generator().manual_seed(sum(shape))
    g = (0.95 + 0.05 * torch.rand(shape, generator=gen)).to(dtype).pin_memory()
    x = torch.randn(shape, generator=gen).to(dtype).pin_memory()
    go = torch.randn(shape, generator=gen).to(dtype).pin_memory()
    y, dg, dt = scan_fwd_bwd_host(g, x, go, block_bytes=block_bytes, depth=depth)
    gd, xd, god = g.cuda(), x.cuda(), go.cuda()
    yd = fp.scan_forward(gd, xd)
    dgd, dtd = fp.scan_backward(gd, yd, god)
    import oracle

    tol = 1e-5 if dtype == torch.float32 else 1e-2
    for a, b in ((y, yd), (dt, dtd), (dg, dgd)):
        assert oracle.normwise_error(a.double().numpy(), b.double().cpu().numpy()) <= tol


def test_offload_rejects_device_tensors():
    t = torch.rand(1, 1, 32, device="cuda")
    with pytest.raises(RuntimeError):
        scan_fwd_bwd_host(t, t, t)
