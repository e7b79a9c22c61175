"""BN + activation training forward from statistics its producer computed (the consumer half of
conv-epilogue statistics): a convolution's GEMM epilogue sees the output tile by tile (rows =
output pixels b*S + s, 128 per tile here) and can leave one (count, mean, M2) per tile and
channel; dnb_bn_act_forward_from_stats merges them and applies the layer in one pass over x.

Checks: the merged statistics against float64 over the whole channel and against the reference's
own float32 statistics (the bars of test_gpu_bn.py); the rolling statistics, x_norm and y
bit-identical to the reference op sequence given the kernel's statistics; a piece with count 0 is
skipped."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from darknet_zig_b200 import gpu, synth
from parity import assert_bitexact, assert_close
from test_gpu_bn import check_forward_stats, oracle_bn_apply

pytestmark = pytest.mark.gpu

TILE = 128


def epilogue_pieces(x, B, C, S):
    """[pieces][C][3] (count, mean, M2) over tiles of TILE consecutive output pixels (b*S + s),
    float64, as a GEMM epilogue would leave them; one extra empty piece at the end."""
    xc = x.reshape(B, C, S).transpose(1, 0, 2).reshape(C, B * S).astype(np.float64)
    n = B * S
    P = -(-n // TILE)
    out = np.zeros((P + 1, C, 3), np.float64)
    for p in range(P):
        t = xc[:, p * TILE:min(n, (p + 1) * TILE)]
        m = t.mean(axis=1)
        out[p, :, 0] = t.shape[1]
        out[p, :, 1] = m
        out[p, :, 2] = ((t - m[:, None]) ** 2).sum(axis=1)
    out[P, :, 1] = 1.0e30  # an empty piece: its mean must not count
    return out


def test_an_empty_first_piece_is_skipped(cuda, oracle):
    B, C, S = 8, 16, 64
    x = synth.normal(81, (B * C * S,), 3.0, 1.0)
    pieces = epilogue_pieces(x, B, C, S)
    pieces = np.concatenate([pieces[-1:], pieces[:-1]])  # the empty piece first
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    y = torch.empty(x.size, dtype=torch.float32, device="cuda")
    mean, var, rm, rv = (torch.zeros(C, device="cuda") for _ in range(4))
    g, b = torch.ones(C, device="cuda"), torch.zeros(C, device="cuda")
    gpu.bnActForwardFromStats(d(x), y, None, B, C, S, d(pieces), pieces.shape[0], g, b, mean, var, rm, rv, gpu.LEAKY)
    torch.cuda.synchronize()
    check_forward_stats(oracle, x.copy(), (B, C, S), mean.cpu().numpy(), var.cpu().numpy())


@pytest.mark.parametrize("shape", [(8, 16, 64), (4, 17, 53), (16, 40, 196), (128, 256, 784)])
@pytest.mark.parametrize("act", [gpu.LEAKY, gpu.LINEAR])
def test_forward_from_epilogue_statistics(cuda, oracle, shape, act):
    B, C, S = shape
    x = synth.normal(61, (B * C * S,), 0.4, 1.0)
    gamma = synth.uniform(62, (C,), 0.5, 1.5)
    beta = synth.normal(63, (C,), 0.0, 0.1)
    rm0 = synth.normal(64, (C,), 0.0, 0.5)
    rv0 = synth.uniform(65, (C,), 0.5, 2.0)
    pieces = epilogue_pieces(x, B, C, S)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    y = torch.empty(x.size, dtype=torch.float32, device="cuda")
    xn = torch.empty_like(y)
    mean, var = torch.zeros(C, device="cuda"), torch.zeros(C, device="cuda")
    rm, rv = d(rm0), d(rv0)
    gpu.bnActForwardFromStats(d(x), y, xn, B, C, S, d(pieces), pieces.shape[0], d(gamma), d(beta), mean, var, rm, rv,
                              act)
    torch.cuda.synchronize()
    m_got, v_got = mean.cpu().numpy(), var.cpu().numpy()
    check_forward_stats(oracle, x.copy(), shape, m_got, v_got)
    rm_w, rv_w = rm0.copy(), rv0.copy()
    oracle.scal(0.99, rm_w)
    oracle.axpy(np.float32(1) - np.float32(0.99), m_got, rm_w)
    oracle.scal(0.99, rv_w)
    oracle.axpy(np.float32(1) - np.float32(0.99), v_got, rv_w)
    assert_bitexact(rm.cpu().numpy(), rm_w, "rolling_mean")
    assert_bitexact(rv.cpu().numpy(), rv_w, "rolling_variance")
    xn_w, y_w = oracle_bn_apply(oracle, x, m_got, v_got, gamma, beta, shape, act)
    assert_bitexact(xn.cpu().numpy(), xn_w, "x_norm")
    assert_bitexact(y.cpu().numpy(), y_w, "y")


def test_matches_the_fused_forward_statistics(cuda):
    """The same statistics as the fused forward's own pass, within the reduction bar."""
    B, C, S = 32, 64, 196
    x = synth.normal(71, (B * C * S,), 1.0, 2.0)
    xd = torch.from_numpy(x).cuda()
    g, b = torch.ones(C, device="cuda"), torch.zeros(C, device="cuda")
    y = torch.empty_like(xd)
    m1, v1, m2, v2 = (torch.zeros(C, device="cuda") for _ in range(4))
    z = [torch.zeros(C, device="cuda") for _ in range(4)]
    gpu.bnActForwardTrain(xd, y, None, B, C, S, g, b, m1, v1, z[0], z[1], gpu.LEAKY)
    pieces = torch.from_numpy(epilogue_pieces(x, B, C, S)).cuda()
    gpu.bnActForwardFromStats(xd, y, None, B, C, S, pieces, pieces.shape[0], g, b, m2, v2, z[2], z[3], gpu.LEAKY)
    torch.cuda.synchronize()
    assert_close(m2.cpu().numpy(), m1.cpu().numpy(), "mean", atol=1e-6)
    assert_close(v2.cpu().numpy(), v1.cpu().numpy(), "variance", atol=1e-6)
