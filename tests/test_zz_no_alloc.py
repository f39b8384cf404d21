"""The no-allocation MoE entry point (riallm_cuda_moe_forward_noalloc).

It exists for callers that cannot allocate device memory themselves (their
host owns all device memory, or they must not call into cudaMalloc), so it
takes scratch from an array compiled into the library instead. This test
calls it through the C ABI twice in a row and checks each result against the
regular entry point (riallm_cuda_moe_forward) on the same inputs, checks that
riallm_cuda_moe_forward_noalloc_sync reports clean completion, covers NF4 and
8-bit experts and a call large enough that the expert GEMM runs without its
split-tile workspace, and checks that a call too large for the array is
refused. It sits in a file of its own that pytest collects last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-2  # bf16 activations: max |a - b| / max |b|


def _layer(rb, H, I, E, seed, qtype):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    d = {}
    for name, shape in (("mlp.gate.weight", (E, H)), ("mlp.experts.gate_up_proj", (E, 2 * I, H)),
                        ("mlp.experts.down_proj", (E, H, I))):
        w = torch.empty(shape, device="cuda").normal_(0.0, 0.02, generator=gen)
        d[name] = rb.quantize_tensor(w, qtype)
    return d


@pytest.mark.parametrize("H,I,E,k,T,qt", [
    (512, 512, 8, 2, 24, 1),
    (4096, 14336, 8, 2, 64, 1),
    (4096, 14336, 8, 2, 64, 2),     # 8-bit expert weights
    (4096, 14336, 8, 2, 200, 1),    # 400 pairs: the layout without the split-tile workspace
])
def test_noalloc_matches_regular_entry_point(rb, H, I, E, k, T, qt):
    L = rb.lib()
    d = _layer(rb, H, I, E, seed=H + T + qt, qtype=rb.CompressionType(qt))
    w, keep, _ = rb._weights(d)
    gen = torch.Generator(device="cuda").manual_seed(T)
    x = torch.empty(T, H, device="cuda").normal_(0, 1, generator=gen).to(torch.bfloat16)
    ref = rb.apply_moe(d, x, k, E)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out = torch.full_like(x, float("nan"))
        rc = L.riallm_cuda_moe_forward_noalloc(ctypes.byref(w), x.data_ptr(), out.data_ptr(),
                                               T, H, I, E, k, 0, stream)
        assert rc == 0, rc
        assert L.riallm_cuda_moe_forward_noalloc_sync(stream) == 0  # every wait completed
        err = ((out.float() - ref.float()).abs().max() / ref.float().abs().max()).item()
        assert err < TOL, (call, err)
    del keep


def test_noalloc_refuses_calls_beyond_its_scratch(rb):
    L = rb.lib()
    H, I, E, k = 4096, 14336, 8, 2
    d = _layer(rb, H, I, E, seed=5, qtype=rb.CompressionType.FourBit)
    w, keep, _ = rb._weights(d)
    T = 512  # 1024 token-expert pairs need more than the 24 MiB array
    x = torch.zeros(T, H, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros_like(x)
    stream = torch.cuda.current_stream().cuda_stream
    rc = L.riallm_cuda_moe_forward_noalloc(ctypes.byref(w), x.data_ptr(), out.data_ptr(), T, H, I, E, k, 0,
                                           stream)
    assert rc == 1  # RIALLM_ERR_MEMORY: refused before launching anything
    assert L.riallm_cuda_moe_forward_noalloc_sync(stream) == 0
    assert torch.count_nonzero(out).item() == 0
    # A wrong element count is a configuration error, as in the regular entry point.
    bad = rb.CMoeWeights.from_buffer_copy(w)
    bad.down_proj.numel -= 1
    assert L.riallm_cuda_moe_forward_noalloc(ctypes.byref(bad), x.data_ptr(), out.data_ptr(), 4, H, I, E, k, 0,
                                             stream) == 3
    del keep
