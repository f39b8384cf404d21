"""Failure detection on the GPU without a fault: a bounded device-side wait
made to expire (a partial-sum count that no CTA reaches, through the
riallm_cuda_ctx_expire_next_wait test hook) must come back as
RIALLM_ERR_TIMEOUT from riallm_cuda_stream_synchronize within the
configured bound, and the same context must then compute correctly."""
import time

import numpy as np
import pytest
import torch

from conftest import rel_err
from test_gpu_moe import dev_tensors, set_shapes, to_dev_x

pytestmark = pytest.mark.gpu


def test_expired_wait_reports_timeout_and_context_recovers(rb, oracle_lib):
    O = oracle_lib
    H, I, E, k, T = 4096, 1024, 8, 2, 8  # few tiles: every one is cut across CTAs
    w, _ = O.synthetic_layer(H, I, E, 1, seed=21)
    x = O.synthetic_x(T, H, seed=22)
    ref, *_ = O.moe_forward(w, x, T, H, I, E, k)
    d = set_shapes(dev_tensors(rb, w), H, I, E)
    xt = to_dev_x(x, True)
    ctx = rb.Context(0)
    try:
        good = rb.apply_moe(d, xt, k, E, ctx=ctx)
        ctx.synchronize()
        assert rel_err(good.float().cpu().numpy(), ref) < 2e-2
        ctx.set_wait_limit(2_000_000)  # 2 ms
        ctx.expire_next_wait()
        t0 = time.time()
        rb.apply_moe(d, xt, k, E, ctx=ctx)
        with pytest.raises(rb.TimeoutError_):
            ctx.synchronize()
        assert time.time() - t0 < 5.0
        # The same context recovers: identical bits to the good call.
        again = rb.apply_moe(d, xt, k, E, ctx=ctx)
        ctx.synchronize()
        assert torch.equal(again, good)
        ctx.set_wait_limit(0)
        with pytest.raises(rb.ConfigError):
            ctx.set_wait_limit(10)
    finally:
        torch.cuda.synchronize()
        ctx.close()
