"""Expert-parallel MoE on the GPU: the ranks' float32 partials
(riallm_cuda_moe_forward_ep over expert slices) must sum to the whole block,
and ExpertParallelMoE over NCCL must reproduce the single-GPU block when two
GPUs are present."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _layer(rb, H, I, E, qt, seed, dev):
    gen = torch.Generator(device=dev).manual_seed(seed)
    d = {}
    for name, shape in [("mlp.gate.weight", (E, H)), ("mlp.experts.gate_up_proj", (E, 2 * I, H)),
                        ("mlp.experts.down_proj", (E, H, I))]:
        w = torch.empty(shape, device=dev).normal_(0.0, 0.02, generator=gen)
        d[name] = rb.quantize_tensor(w, rb.CompressionType(qt))
    return d, gen


def _local(d, e_begin, e_local):
    return {"mlp.gate.weight": d["mlp.gate.weight"],
            "mlp.experts.gate_up_proj": d["mlp.experts.gate_up_proj"].expert_slice(e_begin, e_local),
            "mlp.experts.down_proj": d["mlp.experts.down_proj"].expert_slice(e_begin, e_local)}


@pytest.mark.parametrize("H,I,E,k,T,qt,W", [(512, 512, 8, 2, 40, 1, 2), (512, 768, 8, 2, 40, 1, 4),
                                             (1024, 512, 16, 4, 33, 2, 4), (512, 512, 8, 2, 300, 1, 8)])
def test_partials_sum_to_block(rb, H, I, E, k, T, qt, W):
    dev = torch.device("cuda", 0)
    d, gen = _layer(rb, H, I, E, qt, seed=H + E + T, dev=dev)
    x = torch.empty(T, H, device=dev).normal_(0, 1, generator=gen).to(torch.bfloat16)
    full = rb.apply_moe(d, x, k, E).float()
    total = torch.zeros(T, H, device=dev)
    for r in range(W):
        e_b, e_l = r * E // W, E // W
        total += rb.apply_moe_ep_partial(_local(d, e_b, e_l), x, k, E, e_b, e_l)
    torch.cuda.synchronize()
    err = rel_err(total.to(torch.bfloat16).float().cpu().numpy(), full.cpu().numpy())
    assert err < 5e-3, err


def test_ep_argument_errors(rb):
    dev = torch.device("cuda", 0)
    d, gen = _layer(rb, 512, 512, 8, 1, seed=1, dev=dev)
    x = torch.zeros(4, 512, device=dev, dtype=torch.bfloat16)
    with pytest.raises(rb.ConfigError):
        rb.apply_moe_ep_partial(_local(d, 6, 2), x, 2, 8, 6, 4)  # range past E
    with pytest.raises(rb.ConfigError):
        d["mlp.experts.gate_up_proj"].expert_slice(7, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, result_dir):
    import datetime
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import riallm_b200 as rb
    from riallm_b200.ep import ExpertParallelMoE, expert_range
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        bad, rels = 0, []
        from riallm_b200.ep import ExpertParallelA2A
        # (H, I, E, k, T): 4 experts per rank; 16 experts per rank (16
        # segments per peer in the reorders).
        for case, (H, I, E, k, T) in enumerate(((1024, 1024, 8, 2, 24), (512, 256, 32, 4, 40))):
            d, gen = _layer(rb, H, I, E, 1, seed=5 + case, dev=dev)
            x_all = torch.empty(world * T, H, device=dev).normal_(0, 1, generator=gen).to(torch.bfloat16)
            full = rb.apply_moe(d, x_all, k, E).float()
            e_b, e_l = expert_range(E, rank, world)
            mine = full[rank * T:(rank + 1) * T]
            outs = []
            if case == 0:
                blk = ExpertParallelMoE(_local(d, e_b, e_l), E, k)
                outs.append(blk(x_all[rank * T:(rank + 1) * T]))
            # The token all-to-all inside the library, twice (the second call
            # reuses the communicator and the receive arena).
            a2a = ExpertParallelA2A(_local(d, e_b, e_l), E, k, device=rank)
            for _ in range(2):
                outs.append(a2a(x_all[rank * T:(rank + 1) * T]))
            torch.cuda.synchronize()
            a2a.close()
            # The peer-memory transport: rows stored into the other GPU's
            # mapped buffers by the library's kernels, three calls in a row.
            peer = ExpertParallelA2A(_local(d, e_b, e_l), E, k, device=rank, transport="peer", max_tokens=T)
            for _ in range(3):
                outs.append(peer(x_all[rank * T:(rank + 1) * T]))
            torch.cuda.synchronize()
            peer.ctx.synchronize()
            peer.close()
            for o in outs:
                b_, r_ = _bf16_bound(o.float(), mine)
                bad += b_
                rels.append(r_)
        with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
            f.write(f"{bad} {max(rels)}\n")
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _bf16_bound(a, b):
    """(elements beyond one bf16 ulp + 1e-3 max|b|, max|a-b| / max|b|): the
    expert-parallel block sums the same float32 terms as the single-GPU one in
    another order and rounds each output to bf16 once, so an element may
    differ by one rounding step."""
    diff = (a - b).abs()
    _, ex = torch.frexp(torch.maximum(a.abs(), b.abs()))
    ulp = torch.ldexp(torch.ones_like(diff), (ex - 8).to(torch.int32))
    scale = b.abs().max()
    return int((diff > ulp + 1e-3 * scale).sum()), float(diff.max() / scale)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_expert_parallel_nccl_two_gpus(tmp_path):
    mp.spawn(_nccl_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    for r in range(2):
        bad, rel = open(tmp_path / f"rank{r}.txt").read().split()
        assert int(bad) == 0 and float(rel) < 1e-2, (bad, rel)
