"""Layer glue kernels vs the reference torch sequence (models/tensor_ops.py)."""

import pytest
import torch

from cxlsparse_b200 import _lib
from cxlsparse_b200.model import rms_norm, rotary

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


@pytest.mark.parametrize("dim", [2048, 8192, 1000, 9000])  # vector path, then scalar
def test_rms_norm_matches_torch_sequence(cuda, dim):
    torch.manual_seed(0)
    x = torch.randn(37, dim, device=cuda).bfloat16()
    w = (torch.rand(dim, device=cuda) + 0.5).bfloat16()
    out = torch.empty_like(x)
    _lib.check(_lib.lib().cxs_rms_norm(x.data_ptr(), w.data_ptr(), out.data_ptr(), 37, dim,
                                       1e-6, _stream()))
    torch.testing.assert_close(out.float(), rms_norm(x, w, 1e-6).float(), rtol=0.01, atol=0.01)


def test_residual_rms_norm_matches_add_then_norm(cuda):
    """hidden += delta in bf16 (kept as the new residual), then RMSNorm of the
    sum: the reference's residual add followed by the next norm."""
    torch.manual_seed(3)
    rows, dim = 256, 2048
    hidden = torch.randn(rows, dim, device=cuda).bfloat16()
    delta = (0.1 * torch.randn(rows, dim, device=cuda)).bfloat16()
    w = (torch.rand(dim, device=cuda) + 0.5).bfloat16()
    expect_h = hidden + delta
    expect = rms_norm(expect_h, w, 1e-6)
    out = torch.empty_like(hidden)
    _lib.check(_lib.lib().cxs_residual_rms_norm(hidden.data_ptr(), delta.data_ptr(), w.data_ptr(),
                                                out.data_ptr(), rows, dim, 1e-6, _stream()))
    assert torch.equal(hidden, expect_h)  # the bf16 sum, bit for bit
    torch.testing.assert_close(out.float(), expect.float(), rtol=0.01, atol=0.01)
    with pytest.raises(ValueError, match="multiple of 8"):
        _lib.check(_lib.lib().cxs_residual_rms_norm(hidden.data_ptr(), delta.data_ptr(),
                                                    w.data_ptr(), out.data_ptr(), rows, 1000 + 4,
                                                    1e-6, _stream()))


def test_qkv_rope_gates_and_packing(cuda):
    torch.manual_seed(1)
    E, qh, kvh = 40, 32, 2
    proj = torch.randn(E, qh * 64 + 2 * kvh * 64 + qh * 3, device=cuda).bfloat16()
    positions = torch.arange(1000, 1000 + E, device=cuda, dtype=torch.int32)
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, 64, 2, device=cuda).float() / 64))
    query = torch.empty(E, qh, 64, dtype=torch.bfloat16, device=cuda)
    window = torch.zeros(5 + E, kvh, 128, dtype=torch.bfloat16, device=cuda)
    current = torch.empty(kvh, E, 128, dtype=torch.bfloat16, device=cuda)
    gates = torch.empty(E, qh * 3, dtype=torch.bfloat16, device=cuda)
    _lib.check(_lib.lib().cxs_qkv_rope(
        proj.data_ptr(), proj.shape[1], positions.data_ptr(), inv_freq.data_ptr(), E, qh, kvh,
        query.data_ptr(), window[5:].data_ptr(), kvh * 128, current.data_ptr(), E * 128,
        gates.data_ptr(), _stream()))
    q = proj[:, : qh * 64].view(E, qh, 64)
    k = proj[:, qh * 64: qh * 64 + kvh * 64].view(E, kvh, 64)
    v = proj[:, qh * 64 + kvh * 64: qh * 64 + 2 * kvh * 64].view(E, kvh, 64)
    g = torch.sigmoid(proj[:, qh * 64 + 2 * kvh * 64:])
    rq, rk = rotary(q, k, positions.long(), inv_freq)
    records = torch.cat((rk, v), -1)
    torch.testing.assert_close(query.float(), rq.float(), rtol=0.016, atol=0.016)
    torch.testing.assert_close(window[5:].float(), records.float(), rtol=0.016, atol=0.016)
    assert window[:5].eq(0).all()
    torch.testing.assert_close(current.transpose(0, 1).float(), records.float(), rtol=0.016,
                               atol=0.016)
    torch.testing.assert_close(gates.float(), g.float(), rtol=0.01, atol=0.01)


@pytest.mark.parametrize("ffn", [300, 5632])  # scalar path, vector path
def test_silu_mul(cuda, ffn):
    torch.manual_seed(2)
    gu = torch.randn(9, 2 * ffn, device=cuda).bfloat16()
    out = torch.empty(9, ffn, dtype=torch.bfloat16, device=cuda)
    _lib.check(_lib.lib().cxs_silu_mul(gu.data_ptr(), 9, ffn, out.data_ptr(), _stream()))
    expected = torch.nn.functional.silu(gu[:, :ffn]) * gu[:, ffn:]
    torch.testing.assert_close(out.float(), expected.float(), rtol=0.01, atol=0.01)
