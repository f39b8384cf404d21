"""The peer-memory expert-parallel transport (riallm_cuda_ep_peer_init +
riallm_cuda_moe_forward_ep_peer) on one GPU as a one-rank group: every
"peer" store then lands in this rank's own symmetric buffer, and the plan,
dispatch, return and epoch-flag hand-offs run as they do across GPUs. The
output must match the single-GPU block within one bf16 rounding step per
element (the expert GEMM sums the same terms in another tile schedule),
over several calls in a row (the free/arrived flags of call n wait on
call n - 1) and when a call is replayed from a CUDA graph. Runs in a child
process so the process group does not outlive the test."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bound(a, b):
    diff = (a - b).abs()
    _, ex = torch.frexp(torch.maximum(a.abs(), b.abs()))
    ulp = torch.ldexp(torch.ones_like(diff), (ex - 8).to(torch.int32))
    scale = b.abs().max()
    return int((diff > ulp + 1e-3 * scale).sum()), float(diff.max() / scale)


def _worker(rank, port, result):
    import datetime
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist
    import riallm_b200 as rb
    from riallm_b200.ep import ExpertParallelA2A
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=120), device_id=dev)
    lines = []
    try:
        for case, (H, I, E, k, T, qt) in enumerate(((1024, 1024, 8, 2, 40, 1), (512, 256, 32, 4, 24, 2))):
            gen = torch.Generator(device=dev).manual_seed(11 + case)
            d = {}
            for name, shape in (("mlp.gate.weight", (E, H)), ("mlp.experts.gate_up_proj", (E, 2 * I, H)),
                                ("mlp.experts.down_proj", (E, H, I))):
                w = torch.empty(shape, device=dev).normal_(0.0, 0.02, generator=gen)
                d[name] = rb.quantize_tensor(w, rb.CompressionType(qt))
            x = torch.empty(T, H, device=dev).normal_(0, 1, generator=gen).to(torch.bfloat16)
            ref = rb.apply_moe(d, x, k, E).float()
            blk = ExpertParallelA2A(d, E, k, device=0, transport="peer", max_tokens=T)
            outs = [blk(x) for _ in range(3)]
            # A smaller call fits the same set-up.
            small = blk(x[: T // 2])
            torch.cuda.synchronize()
            blk.ctx.synchronize()
            for o in outs:
                lines.append(("eager", case) + _bound(o.float(), ref))
            lines.append(("small", case) + _bound(small.float(), rb.apply_moe(d, x[: T // 2], k, E).float()))
            # One call captured in a graph, replayed twice.
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                blk(x)
            torch.cuda.current_stream().wait_stream(side)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                gout = blk(x)
            for _ in range(2):
                g.replay()
            torch.cuda.synchronize()
            blk.ctx.synchronize()
            lines.append(("graph", case) + _bound(gout.float(), ref))
            del g
            blk.close()
        with open(result, "w") as f:
            for ln in lines:
                f.write(" ".join(str(v) for v in ln) + "\n")
    finally:
        dist.destroy_process_group()


def test_peer_transport_one_rank_matches_block(tmp_path):
    out = str(tmp_path / "r.txt")
    mp.spawn(_worker, args=(_free_port(), out), nprocs=1, join=True)
    rows = [ln.split() for ln in open(out).read().splitlines()]
    assert len(rows) == 10
    for kind, case, bad, rel in rows:
        assert int(bad) == 0 and float(rel) < 1e-2, (kind, case, bad, rel)
