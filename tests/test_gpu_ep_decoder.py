"""The expert-parallel decoder (Decoder(ep=ExpertParallelMoE)) against the
plain decoder, on one GPU as a one-rank NCCL group: the all-gather and the
reduce-scatter are then identities, the rank holds every expert, and the
decode step (collectives included) is captured in the decode graph. The
block output is added to the residual stream in float32 and rounded once on
both paths, so greedy tokens must agree and logits stay within 2e-2 (the
tiny configuration, synthetic weights seed 0). Runs in a child process so
the process group does not outlive the test."""
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


def _worker(rank, port, result):
    import datetime
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch.distributed as dist
    from riallm_b200 import decoder as D
    from riallm_b200.ep import ExpertParallelMoE
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(0)
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", 0))
    try:
        cfg = D.DecoderConfig()
        qw = D.synthetic_model(cfg, seed=0, device="cuda")
        g = torch.Generator().manual_seed(1)
        prompt = torch.randint(0, cfg.vocab, (2, 24), generator=g).cuda()
        plain = D.Decoder(cfg, qw, max_batch=2, max_seq=64)
        t0, l0 = plain.generate(prompt, 8, keep_logits=True)
        plain.close()
        ep = ExpertParallelMoE(None, cfg.experts, cfg.top_k)
        par = D.Decoder(cfg, qw, max_batch=2, max_seq=64, ep=ep)
        t1, l1 = par.generate(prompt, 8, keep_logits=True)
        par.close()
        torch.cuda.synchronize()
        err = float((l1 - l0).abs().max() / l0.abs().max())
        same = bool(torch.equal(t0, t1))
        with open(result, "w") as f:
            f.write(f"{int(same)} {err}\n")
    finally:
        dist.destroy_process_group()


def test_expert_parallel_decoder_matches_plain(tmp_path):
    out = str(tmp_path / "r.txt")
    mp.spawn(_worker, args=(_free_port(), out), nprocs=1, join=True)
    same, err = open(out).read().split()
    assert float(err) < 2e-2, err
    assert same == "1"
