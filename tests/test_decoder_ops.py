"""The element-wise decoder kernels against the reference's host restatements (oracle): lb_qkv_prep
(hub_gpu.py:1701-1723: split, optional per-head RMSNorm, half-split rotary, cache write) and lb_act_mul
(hub_gpu.py:1755-1762: silu / tanh-gelu gate times up).  Outputs are bf16, so they are compared within one
bf16 rounding of the float32 oracle on the same (bf16) inputs."""
import numpy as np
import pytest
import torch

from oracle import lowbit_oracle as O

pytestmark = pytest.mark.gpu


def _within_bf16(got, ref, slack=1e-6):
    got, ref = np.asarray(got, np.float32), np.asarray(ref, np.float32)
    return np.all(np.abs(got - ref) <= np.abs(ref) * 2.0 ** -7 + slack)


@pytest.mark.parametrize("norm", [False, True])
@pytest.mark.parametrize("rot", [64, 40])
def test_qkv_prep_matches_reference(cuda, norm, rot):
    from apsi_b200 import kernels as Kn
    B, T, nh, kvh, dh, cap, start = 2, 3, 4, 2, 64, 16, 5
    g = torch.Generator(device=cuda).manual_seed(7)
    qkv = torch.randn((B * T, (nh + 2 * kvh) * dh), generator=g, device=cuda).to(torch.bfloat16)
    half = rot // 2
    inv = 1.0 / (10000.0 ** (torch.arange(half, device=cuda, dtype=torch.float32) / half))
    ang = torch.arange(cap, device=cuda, dtype=torch.float32)[:, None] * inv[None]
    cos, sin = torch.cos(ang).contiguous(), torch.sin(ang).contiguous()
    qn = (torch.rand(dh, generator=g, device=cuda) + 0.5).to(torch.bfloat16) if norm else None
    kn = (torch.rand(dh, generator=g, device=cuda) + 0.5).to(torch.bfloat16) if norm else None
    q = torch.zeros((B, nh, T, dh), dtype=torch.bfloat16, device=cuda)
    kc = torch.full((B, kvh, cap, dh), 7.0, dtype=torch.bfloat16, device=cuda)
    vc = torch.full((B, kvh, cap, dh), 7.0, dtype=torch.bfloat16, device=cuda)
    Kn.qkv_prep(qkv, B, T, nh, kvh, dh, rot, cos, sin, q, kc, vc, start=start, qn=qn, kn=kn, eps=1e-6)
    torch.cuda.synchronize(cuda)
    x = qkv.float().cpu().numpy().reshape(B, T, -1)
    for b in range(B):
        rq, rk, rv = O.qkv_prep(x[b], cos.cpu().numpy(), sin.cpu().numpy(),
                                None if qn is None else qn.float().cpu().numpy(),
                                None if kn is None else kn.float().cpu().numpy(), nh, kvh, dh, rot, start, 1e-6)
        assert _within_bf16(q[b].float().cpu().numpy().transpose(1, 0, 2), rq)
        assert _within_bf16(kc[b, :, start:start + T].float().cpu().numpy().transpose(1, 0, 2), rk)
        assert np.array_equal(vc[b, :, start:start + T].float().cpu().numpy().transpose(1, 0, 2), rv)
    # cache positions outside [start, start + T) are untouched
    assert torch.all(kc[:, :, :start] == 7.0) and torch.all(kc[:, :, start + T:] == 7.0)
    # positions from a device scalar land in the same place
    kc2 = torch.full_like(kc, 7.0)
    vc2 = torch.full_like(vc, 7.0)
    q2 = torch.zeros_like(q)
    Kn.qkv_prep(qkv, B, T, nh, kvh, dh, rot, cos, sin, q2, kc2, vc2, pos0=torch.tensor([start], device=cuda),
                qn=qn, kn=kn, eps=1e-6)
    assert torch.equal(q2, q) and torch.equal(kc2, kc) and torch.equal(vc2, vc)


@pytest.mark.parametrize("kind", [0, 1])
@pytest.mark.parametrize("I", [512, 100])
def test_act_mul_matches_reference(cuda, kind, I):
    from apsi_b200 import kernels as Kn
    g = torch.Generator(device=cuda).manual_seed(kind + I)
    gu = (torch.randn((5, 2 * I), generator=g, device=cuda) * 3).to(torch.bfloat16)
    out = Kn.act_mul(gu, I, kind)
    ref = O.act_mul(gu.float().cpu().numpy(), I, kind)
    assert _within_bf16(out.float().cpu().numpy(), ref, slack=1e-5)
