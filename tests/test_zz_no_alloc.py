"""The no-allocation MoE entry point (riallm_cuda_moe_forward_noalloc).

It exists for callers that cannot allocate device memory themselves (their
host owns all device memory, or they must not call into cudaMalloc), so it
takes scratch from an array compiled into the library instead. This test
calls it through the C ABI twice in a row and checks each result against the
regular entry point (riallm_cuda_moe_forward) on the same inputs, and checks
that a call too large for the array is refused. It sits in a file of its own
that pytest collects last.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 2e-2  # bf16 activations: max |a - b| / max |b|


def _layer(rb, H, I, E, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    d = {}
    for name, shape in (("mlp.gate.weight", (E, H)), ("mlp.experts.gate_up_proj", (E, 2 * I, H)),
                        ("mlp.experts.down_proj", (E, H, I))):
        w = torch.empty(shape, device="cuda").normal_(0.0, 0.02, generator=gen)
        d[name] = rb.quantize_tensor(w, rb.CompressionType.FourBit)
    return d


@pytest.mark.parametrize("H,I,E,k,T", [(512, 512, 8, 2, 24), (4096, 14336, 8, 2, 64)])
def test_noalloc_matches_regular_entry_point(rb, H, I, E, k, T):
    L = rb.lib()
    d = _layer(rb, H, I, E, seed=H + T)
    w, keep, _ = rb._weights(d)
    x = torch.empty(T, H, device="cuda").normal_(0, 1).to(torch.bfloat16)
    ref = rb.apply_moe(d, x, k, E)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):
        out = torch.full_like(x, float("nan"))
        rc = L.riallm_cuda_moe_forward_noalloc(ctypes.byref(w), x.data_ptr(), out.data_ptr(),
                                               T, H, I, E, k, 0, stream)
        assert rc == 0, rc
        torch.cuda.synchronize()
        err = ((out.float() - ref.float()).abs().max() / ref.float().abs().max()).item()
        assert err < TOL, (call, err)
    del keep


def test_noalloc_refuses_calls_beyond_its_scratch(rb):
    L = rb.lib()
    H, I, E, k = 4096, 14336, 8, 2
    d = _layer(rb, H, I, E, seed=5)
    w, keep, _ = rb._weights(d)
    T = 512  # 1024 token-expert pairs need more than the 24 MiB array
    x = torch.zeros(T, H, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros_like(x)
    rc = L.riallm_cuda_moe_forward_noalloc(ctypes.byref(w), x.data_ptr(), out.data_ptr(), T, H, I, E, k, 0,
                                           torch.cuda.current_stream().cuda_stream)
    assert rc == 1  # RIALLM_ERR_MEMORY: refused before launching anything
    assert torch.count_nonzero(out).item() == 0
    del keep
