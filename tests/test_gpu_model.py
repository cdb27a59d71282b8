"""GPU: the RansLinear layer (fused decode-GEMV + escape corrections) and the
encoded-matrix container, against float64 references on the same codes."""
import numpy as np
import pytest

from oracle import rans_oracle as orc
import rans_model as rm

pytestmark = pytest.mark.gpu
REL_L2 = 1e-3


@pytest.fixture(scope="module")
def torch(cuda_ok):
    import torch as t
    import rans_b200
    rans_b200.load()
    return t


def _case(rows, cols, bits, seed):
    rng = np.random.default_rng(seed)
    W = rng.standard_t(2.0, (rows, cols)) * 0.01
    codes, step = rm.ecsq_rtn(W, bits)
    return codes, step


@pytest.mark.parametrize("rows,cols,bits", [(256, 1536, 6.5), (1536, 1536, 3.25), (512, 8960, 5.0)])
def test_rans_linear_gemv_with_escapes(torch, rows, cols, bits):
    codes, step = _case(rows, cols, bits, rows + cols)
    C = 640 if cols == 8960 else 512
    m = rm.EncodedMatrix.encode(codes, step, R=8, C=C)
    lin = rm.RansLinear(m)
    x = torch.randn(cols).bfloat16()
    yref = orc.gemv(codes.astype(np.int64), step.astype(np.float64), x.float().numpy().astype(np.float64))
    y = lin(x.cuda()).float().cpu().numpy()               # bf16 output
    assert orc.rel_l2(y, yref) < 1e-2
    yf = lin.gemv(x.cuda()).cpu().numpy()                 # fp32 output
    assert orc.rel_l2(yf, yref) <= REL_L2
    if bits >= 5.0:
        assert lin.n_escapes > 0


def test_rans_linear_dense_weight_and_batch(torch):
    codes, step = _case(512, 1536, 6.5, 7)
    m = rm.EncodedMatrix.encode(codes, step, R=8, C=512)
    assert m.n_escapes > 0
    bias = torch.randn(512)
    lin = rm.RansLinear(m, bias=bias)
    w = lin.weight_bf16().cpu()
    want = (torch.from_numpy(codes).float() * torch.from_numpy(step)).bfloat16()
    assert torch.equal(w, want)                            # escapes included, bit-exact
    x = torch.randn(3, 1536).bfloat16()
    y = lin(x.cuda()).float().cpu()
    yref = x.float() @ want.float().T + bias
    assert (y - yref).norm() / yref.norm() < 1e-2
    y1 = lin(x[:1].cuda()).float().cpu()                   # batch-1 path with bias
    assert (y1 - yref[:1]).norm() / yref[:1].norm() < 1e-2


def test_container_to_layer(torch, tmp_path):
    codes, step = _case(256, 1024, 6.0, 3)
    m = rm.EncodedMatrix.encode(codes, step, R=8, C=512)
    path = str(tmp_path / "w.rans")
    rm.save_matrices(path, {"w": m})
    loaded, _ = rm.load_matrices(path)
    a, b = rm.RansLinear(m), rm.RansLinear(loaded["w"])
    x = torch.randn(1024).bfloat16().cuda()
    # same kernels on the same bytes; only the order of fp32 atomic adds
    # (split column blocks, escapes) may differ between the two calls
    assert orc.rel_l2(a.gemv(x).cpu().numpy(), b.gemv(x).cpu().numpy()) < 1e-6
    assert torch.equal(a.weight_bf16(), b.weight_bf16())


def test_from_weight(torch):
    lin_d = torch.nn.Linear(1536, 256, bias=True)
    lin = rm.RansLinear.from_weight(lin_d.weight, 6.0, bias=lin_d.bias.detach())
    x = torch.randn(1536)
    y = lin.gemv(x.cuda()).cpu() + lin_d.bias.detach()
    yd = lin_d(x.bfloat16().float()).detach()
    # quantisation error at 6 bits/weight stays small against the dense layer
    assert (y - yd).norm() / yd.norm() < 0.05
