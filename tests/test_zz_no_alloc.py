"""rmoe_matmul_mxfp4_noalloc (fixed device scratch, no allocation) against rmoe_matmul_mxfp4 on
the same inputs, two calls in a row, through the C ABI. Collected last so it also runs after
every other GPU test has used the device."""
import numpy as np
import pytest

from oracle import oracle as orc
from refvec import random_vec, rel_l2

pytestmark = pytest.mark.gpu

GEMM_RTOL = 2e-3  # same tolerance as the allocating entry point's parity tests


def _t(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("s,i,o", [(1, 8192, 256), (8, 1024, 96), (512, 8192, 16), (5, 40, 7),
                                   (1030, 4100, 3)])  # (i % 32 != 0: no scratch, no limit)
def test_noalloc_matches_allocating_entry_point(cuda_ctx, s, i, o):
    import torch

    import rabbit_b200 as rb

    w = random_vec(o * i, 3000 + i) * np.float32(4.0)
    q, bs = orc.pack_mxfp4(w, o, i)
    qd, bsd = _t(q), _t(bs)
    for call in range(2):  # second call: new activations through the same scratch
        x = _t(random_vec(s * i, 4000 + 17 * call + s).reshape(s, i))
        want = torch.zeros((s, o), dtype=torch.float32, device="cuda")
        rb.matmul_mxfp4(want, x, qd, bsd, s, i, o)
        got = torch.full((s, o), float("nan"), dtype=torch.float32, device="cuda")
        rb.matmul_mxfp4_noalloc(got, x, qd, bsd, s, i, o)
        torch.cuda.synchronize()
        assert rel_l2(got.cpu().numpy(), want.cpu().numpy()) < GEMM_RTOL


def test_noalloc_rejects_oversize_scratch(cuda_ctx):
    import torch

    import rabbit_b200 as rb

    s, i, o = 513, 8192, 1  # 513*8192 f16 values exceed the fixed 8 MiB + 4 KiB scratch
    y = torch.zeros((s, o), dtype=torch.float32, device="cuda")
    x = torch.zeros((s, i), dtype=torch.float32, device="cuda")
    q = torch.zeros(o * i // 2, dtype=torch.uint8, device="cuda")
    bs = torch.zeros(o * i // 32, dtype=torch.uint8, device="cuda")
    with pytest.raises(rb.RmoeError, match="INVALID_ARG"):
        rb.matmul_mxfp4_noalloc(y, x, q, bs, s, i, o)
