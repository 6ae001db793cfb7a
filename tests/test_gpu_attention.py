"""Causal GQA attention kernels against a plain PyTorch fp32 reference of the
same op (the reference computes it with at::scaled_dot_product_attention on
repeat_interleave'd K/V, layer_forward_impl.inc:41-49): forward output and
log-sum-exp of the tcgen05/TMEM kernel and of the mma.sync kernel, and the
backward (dq, dk, dv) against torch autograd: the tcgen05 kernels at head_dim
128 (64-query items) and 64 (128-query items, one CTA per query head, dK/dV
summed over the GQA heads), and the mma.sync kernels."""
import ctypes as C
import math

import pytest
import torch

from glt_b200 import _lib

pytestmark = pytest.mark.gpu
lib = _lib.lib
TC, MMA = 0, 1


def vp(t):
    return C.c_void_p(t.data_ptr())


def ref_attention(q, k, v, B, T, nh, nkv, hd):
    qh = q.float().view(B, T, nh, hd).transpose(1, 2)
    kh = k.float().view(B, T, nkv, hd).transpose(1, 2).repeat_interleave(nh // nkv, 1)
    vh = v.float().view(B, T, nkv, hd).transpose(1, 2).repeat_interleave(nh // nkv, 1)
    s = (qh @ kh.transpose(-1, -2)) / math.sqrt(hd)
    s = s.masked_fill(~torch.ones(T, T, dtype=torch.bool, device=q.device).tril(), float("-inf"))
    lse = torch.logsumexp(s, -1)                       # [B, nh, T]
    o = torch.softmax(s, -1) @ vh
    return o.transpose(1, 2).reshape(B * T, nh * hd), lse


def make_qkv(B, T, nh, nkv, hd, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    QKV = (nh + 2 * nkv) * hd
    return (torch.randn(B * T, QKV, device="cuda", generator=g) * 1.5).to(torch.bfloat16)


def fwd(qkv, B, T, nh, nkv, hd, impl):
    o = torch.empty(B * T, nh * hd, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B, nh, T, device="cuda")
    _lib.check(lib.glt_attention_fwd(vp(qkv), qkv.shape[1], vp(o), nh * hd, vp(lse), B, T, nh, nkv,
                                     hd, impl, C.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    return o, lse


@pytest.mark.parametrize("impl", [TC, MMA])
@pytest.mark.parametrize("B,T,nh,nkv,hd", [(2, 256, 4, 2, 128), (1, 512, 8, 2, 128),
                                           (2, 256, 4, 4, 64), (1, 384, 6, 2, 64),
                                           (2, 256, 14, 2, 64), (1, 1024, 32, 8, 128)])
def test_forward_matches_fp32_reference(impl, B, T, nh, nkv, hd):
    qkv = make_qkv(B, T, nh, nkv, hd, seed=T + nh + hd)
    q = qkv[:, :nh * hd]
    k = qkv[:, nh * hd:(nh + nkv) * hd]
    v = qkv[:, (nh + nkv) * hd:]
    o, lse = fwd(qkv, B, T, nh, nkv, hd, impl)
    o_ref, lse_ref = ref_attention(q, k, v, B, T, nh, nkv, hd)
    torch.testing.assert_close(o.float(), o_ref, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(lse, lse_ref, rtol=1e-3, atol=1e-3)


def test_tcgen05_and_mma_sync_agree_on_large_scores():
    # large logits exercise the conditional rescale of the tcgen05 kernel
    B, T, nh, nkv, hd = 1, 1024, 4, 1, 128
    qkv = (make_qkv(B, T, nh, nkv, hd, seed=3).float() * 4).to(torch.bfloat16)
    o1, l1 = fwd(qkv, B, T, nh, nkv, hd, TC)
    o2, l2 = fwd(qkv, B, T, nh, nkv, hd, MMA)
    torch.testing.assert_close(o1.float(), o2.float(), rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(l1, l2, rtol=1e-3, atol=2e-3)


@pytest.mark.parametrize("impl,B,T,nh,nkv,hd", [(MMA, 2, 128, 4, 2, 128), (MMA, 1, 256, 4, 4, 64),
                                                (MMA, 2, 256, 14, 2, 64), (MMA, 1, 192, 14, 2, 64),
                                                (TC, 2, 128, 4, 2, 128), (TC, 1, 384, 8, 2, 128),
                                                (TC, 2, 256, 4, 4, 128), (TC, 1, 512, 32, 8, 128),
                                                (TC, 2, 128, 4, 2, 64), (TC, 1, 384, 4, 4, 64),
                                                (TC, 2, 256, 14, 2, 64), (TC, 1, 1024, 14, 2, 64)])
def test_backward_matches_autograd(impl, B, T, nh, nkv, hd):
    qkv = make_qkv(B, T, nh, nkv, hd, seed=11)
    o, lse = fwd(qkv, B, T, nh, nkv, hd, MMA)
    g = torch.Generator(device="cuda").manual_seed(12)
    dout = torch.randn(B * T, nh * hd, device="cuda", generator=g).to(torch.bfloat16)
    dqkv = torch.zeros_like(qkv)
    dq_acc = torch.empty(B * T * (nh + 2 * nkv) * hd, device="cuda")   # dQ (+ dK/dV: tcgen05, hd 64)
    dsum = torch.empty(B * nh * T, device="cuda")
    _lib.check(lib.glt_attention_bwd(vp(qkv), qkv.shape[1], vp(o), vp(dout), nh * hd, vp(lse),
                                     vp(dqkv), vp(dq_acc), vp(dsum), B, T, nh, nkv, hd, impl,
                                     C.c_void_p(torch.cuda.current_stream().cuda_stream)))
    torch.cuda.synchronize()
    x = qkv.float().requires_grad_(True)
    q = x[:, :nh * hd]
    k = x[:, nh * hd:(nh + nkv) * hd]
    v = x[:, (nh + nkv) * hd:]
    o_ref, _ = ref_attention(q, k, v, B, T, nh, nkv, hd)
    o_ref.backward(dout.float())
    ref = x.grad
    for name, sl in (("dq", slice(0, nh * hd)), ("dk", slice(nh * hd, (nh + nkv) * hd)),
                     ("dv", slice((nh + nkv) * hd, None))):
        got, want = dqkv[:, sl].float(), ref[:, sl]
        rel = float((got - want).abs().max() / want.abs().max())
        cos = float(torch.nn.functional.cosine_similarity(got.reshape(-1), want.reshape(-1), dim=0))
        assert rel < 2e-2 and cos > 0.999, (name, rel, cos)
