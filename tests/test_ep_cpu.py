"""Expert-parallel orchestration on CPU: two gloo ranks run
ExpertParallelMoE with a numpy partial-sum function over the oracle's
dequantized weights; every rank's output must match the oracle's whole-block
output for its tokens, and the routing is the oracle's own."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

H, I, E, K, T_LOCAL = 256, 256, 8, 2, 6


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bf16(a):
    from oracle import oracle as O
    return O.bf16_bits_to_f32(O.f32_to_bf16_bits(np.asarray(a, np.float32)))


def _np_partial(O, w, x_all, e_begin, e_local):
    """Sum over each token's pairs with experts in [e_begin, e_begin+e_local),
    expert-ascending, of w * down(silu(gate x) * up x), with the oracle's
    bf16 rounding points (weights and h rounded to bf16)."""
    T = x_all.shape[0]
    wg = O.dequantize(w.gate).reshape(E, H)
    _, _, idx, tw = O.router(x_all, wg, K)
    gu = _bf16(O.dequantize(w.gate_up_proj)).reshape(E, 2 * I, H).astype(np.float64)
    dn = _bf16(O.dequantize(w.down_proj)).reshape(E, H, I).astype(np.float64)
    xf = O.bf16_bits_to_f32(x_all).astype(np.float64)
    out = np.zeros((T, H), np.float32)
    for t in range(T):
        for j in np.argsort(idx[t], kind="stable"):
            e = int(idx[t, j])
            if not (e_begin <= e < e_begin + e_local):
                continue
            g = gu[e, :I] @ xf[t]
            u = gu[e, I:] @ xf[t]
            h = _bf16(g / (1.0 + np.exp(-g)) * u).astype(np.float64)
            y = (dn[e] @ h).astype(np.float32)
            out[t] = out[t] + y * tw[t, j]
    return out


def _worker(rank, world, port, result_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from oracle import oracle as O
    from riallm_b200.ep import ExpertParallelMoE
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w, _ = O.synthetic_layer(H, I, E, 1, seed=11)
        x_all = O.synthetic_x(world * T_LOCAL, H, seed=12, bf16=True)  # bf16 bits [W*T, H]
        ref, idx_ref, _, _ = O.moe_forward(w, x_all, world * T_LOCAL, H, I, E, K)

        def ops(xt, e_begin, e_local):
            bits = xt.view(torch.int16).numpy().view(np.uint16)
            return torch.from_numpy(_np_partial(O, w, bits, e_begin, e_local))

        blk = ExpertParallelMoE({}, E, K, ops=ops)
        assert (blk.e_begin, blk.e_local) == (rank * E // world, E // world)
        x_local = torch.from_numpy(x_all[rank * T_LOCAL:(rank + 1) * T_LOCAL].view(np.int16)).view(torch.bfloat16)
        out = blk(x_local).float().numpy()
        mine = ref[rank * T_LOCAL:(rank + 1) * T_LOCAL]
        err = float(np.abs(out - mine).max() / np.abs(mine).max())
        with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
            f.write(f"{err}\n")
        assert err < 2e-2, err
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_expert_parallel_gloo_matches_oracle(tmp_path, world):
    mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    for r in range(world):
        assert float(open(tmp_path / f"rank{r}.txt").read()) < 2e-2


def test_expert_range_and_slice_rules():
    from riallm_b200.ep import expert_range
    from riallm_b200 import ConfigError
    assert expert_range(8, 3, 4) == (6, 2)
    assert expert_range(128, 7, 8) == (112, 16)
    with pytest.raises(ConfigError):
        expert_range(8, 0, 3)
