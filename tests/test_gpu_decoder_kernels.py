"""The decoder-layer kernels (RMSNorm with the residual add, RoPE + KV-cache
append, cached causal grouped-query attention) against plain torch float32
references of the same ops. Tolerances: outputs are bf16, so 1 bf16 ulp
relative (2^-8) plus float32 reduction-order noise: 1e-2 of max |ref|."""
import math

import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _bf(t):
    return t.to(torch.bfloat16)


@pytest.mark.parametrize("H,rows,with_delta", [(1024, 5, False), (4096, 3, True), (2048, 1, True)])
def test_rmsnorm(rb, H, rows, with_delta):
    from riallm_b200 import Context, lib
    g = torch.Generator(device="cuda").manual_seed(H)
    x = _bf(torch.randn(rows, H, device="cuda", generator=g))
    d = _bf(torch.randn(rows, H, device="cuda", generator=g)) if with_delta else None
    w = torch.rand(H, device="cuda", generator=g) + 0.5
    out = torch.empty_like(x)
    x0 = x.clone()
    ctx = Context.get(0)
    ctx.check(lib().riallm_cuda_rmsnorm(ctx.ptr, x.data_ptr(), d.data_ptr() if d is not None else None,
                                        w.data_ptr(), out.data_ptr(), rows, H, 1e-5,
                                        torch.cuda.current_stream().cuda_stream))
    xr = (x0.float() + d.float()).to(torch.bfloat16) if with_delta else x0
    assert torch.equal(x, xr)  # the residual add is stored, rounded once
    xf = xr.float()
    ref = xf * torch.rsqrt((xf * xf).mean(-1, keepdim=True) + 1e-5) * w
    assert rel_err(out.float().cpu().numpy(), ref.cpu().numpy()) < 1e-2


def _ref_attention(q, kc, vc, pos, T, nh, nkv, d):
    """q [B*T, nh*d]; caches [B, nkv, S, d]; float32 softmax attention of row
    b*T+t over cache positions 0..pos[b]+t."""
    B = kc.shape[0]
    rep = nh // nkv
    out = torch.zeros(B * T, nh * d, device=q.device)
    for b in range(B):
        for t in range(T):
            L = int(pos[b]) + t + 1
            for h in range(nh):
                qq = q[b * T + t, h * d:(h + 1) * d].float()
                k = kc[b, h // rep, :L].float()
                v = vc[b, h // rep, :L].float()
                p = torch.softmax((k @ qq) / math.sqrt(d), 0)
                out[b * T + t, h * d:(h + 1) * d] = p @ v
    return out


# (B, T, positions): small groups split each group's keys over several CTAs;
# B*T*nkv >= 2 * 148 takes the one-CTA-per-group path.
SHAPES = [(3, 4, [0, 9, 600]), (2, 80, [0, 300])]


@pytest.mark.parametrize("nh,nkv,d,shape", [(8, 2, 128, 0), (4, 4, 64, 0), (16, 2, 64, 0), (8, 2, 128, 1),
                                                (48, 8, 128, 0)])
def test_rope_append_and_attention(rb, nh, nkv, d, shape):
    from riallm_b200 import Context, lib
    from riallm_b200.decoder import apply_rope, rope_tables, inv_freq
    B, T, p0 = SHAPES[shape]
    S = 700
    pos = torch.tensor(p0, dtype=torch.int32, device="cuda")  # crosses the 256-key chunks
    g = torch.Generator(device="cuda").manual_seed(nh * 100 + d)
    kc = _bf(torch.randn(B, nkv, S, d, device="cuda", generator=g))
    vc = _bf(torch.randn(B, nkv, S, d, device="cuda", generator=g))
    qkv = _bf(torch.randn(B * T, (nh + 2 * nkv) * d, device="cuda", generator=g))
    q = torch.empty(B * T, nh * d, dtype=torch.bfloat16, device="cuda")
    kc0, vc0 = kc.clone(), vc.clone()
    ctx = Context.get(0)
    st = torch.cuda.current_stream().cuda_stream
    invf = inv_freq(d, 1e6, "cuda")
    ctx.check(lib().riallm_cuda_rope_kv_append(ctx.ptr, qkv.data_ptr(), pos.data_ptr(), B, T, nh, nkv, d,
                                               invf.data_ptr(), q.data_ptr(), kc.data_ptr(), vc.data_ptr(), S, st))
    # torch reference of the rotation and the cache writes
    for b in range(B):
        p = torch.arange(int(pos[b]), int(pos[b]) + T, device="cuda")
        cos, sin = rope_tables(p, d, 1e6)
        rows = qkv[b * T:(b + 1) * T]
        qr = apply_rope(rows[:, :nh * d].view(T, nh, d).transpose(0, 1), cos, sin).transpose(0, 1).reshape(T, -1)
        kr = apply_rope(rows[:, nh * d:(nh + nkv) * d].view(T, nkv, d).transpose(0, 1), cos, sin)
        vr = rows[:, (nh + nkv) * d:].view(T, nkv, d).transpose(0, 1)
        assert rel_err(q[b * T:(b + 1) * T].float().cpu().numpy(), qr.float().cpu().numpy()) < 1e-2
        kc0[b, :, p] = kr
        vc0[b, :, p] = vr
    assert rel_err(kc.float().cpu().numpy(), kc0.float().cpu().numpy()) < 1e-2
    assert torch.equal(vc, vc0)
    out = torch.empty_like(q)
    ctx.check(lib().riallm_cuda_attention(ctx.ptr, q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(),
                                          B, T, nh, nkv, d, S, out.data_ptr(), st))
    ref = _ref_attention(q, kc, vc, pos.cpu(), T, nh, nkv, d)
    assert rel_err(out.float().cpu().numpy(), ref.cpu().numpy()) < 1e-2


def test_argument_errors(rb):
    from riallm_b200 import ConfigError, Context, lib
    ctx = Context.get(0)
    x = torch.zeros(4, 12, dtype=torch.bfloat16, device="cuda")
    w = torch.ones(12, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    with pytest.raises(ConfigError, match="H % 8"):
        ctx.check(lib().riallm_cuda_rmsnorm(ctx.ptr, x.data_ptr(), None, w.data_ptr(), x.data_ptr(), 4, 12, 1e-5, st))
    q = torch.zeros(2, 6 * 128, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(1, 2, 8, 128, dtype=torch.bfloat16, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    with pytest.raises(ConfigError, match="1, 2, 4, 6 or 8"):  # 6 heads over 2 kv heads = 3
        ctx.check(lib().riallm_cuda_attention(ctx.ptr, q.data_ptr(), kc.data_ptr(), kc.data_ptr(), pos.data_ptr(),
                                              1, 2, 6, 2, 128, 8, q.data_ptr(), st))


@pytest.mark.parametrize("M,N,K", [(1, 6144, 4096), (3, 1000, 1024), (8, 4096, 4096), (2, 32000, 256)])
def test_linear_bf16(rb, M, N, K):
    """Skinny bf16 linear layer against a float32 torch matmul of the same
    bf16 inputs (outputs are bf16: 1e-2 of max |ref|)."""
    from riallm_b200 import Context, lib
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    x = _bf(torch.randn(M, K, device="cuda", generator=g))
    w = _bf(torch.randn(N, K, device="cuda", generator=g) * 0.02)
    y = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ctx = Context.get(0)
    ctx.check(lib().riallm_cuda_linear_bf16(ctx.ptr, x.data_ptr(), w.data_ptr(), y.data_ptr(), M, N, K,
                                            torch.cuda.current_stream().cuda_stream))
    ref = x.float() @ w.float().t()
    assert rel_err(y.float().cpu().numpy(), ref.cpu().numpy()) < 1e-2


def test_linear_bf16_errors(rb):
    from riallm_b200 import ConfigError, Context, lib
    ctx = Context.get(0)
    x = torch.zeros(9, 256, dtype=torch.bfloat16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    with pytest.raises(ConfigError, match="M <= 8"):
        ctx.check(lib().riallm_cuda_linear_bf16(ctx.ptr, x.data_ptr(), x.data_ptr(), x.data_ptr(), 9, 256, 256, st))
    with pytest.raises(ConfigError, match="K % 256"):
        ctx.check(lib().riallm_cuda_linear_bf16(ctx.ptr, x.data_ptr(), x.data_ptr(), x.data_ptr(), 1, 2, 200, st))
