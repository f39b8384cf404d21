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
        # add_to: the block's float32 sum is added to a bf16 residual and
        # rounded once, in place (the decoder's residual update).
        g = torch.Generator().manual_seed(40 + rank)
        resid = torch.randn(T_LOCAL, H, generator=g).to(torch.bfloat16)
        y32 = blk._forward(x_local, {}, None)
        want = (resid.float() + y32).to(torch.bfloat16)
        got = blk(x_local, add_to=resid)
        same = bool(got is resid and torch.equal(resid, want))
        with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
            f.write(f"{err}\n")
        assert err < 2e-2, err
        assert same, "add_to must round the float32 sum into the residual once, in place"
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


def _leaver(rank, world, port, result_dir, use_watch):
    """Both ranks take one step; rank 1 then leaves (between steps, nothing
    in flight). Rank 0's next step must raise RankFailureError on the host:
    from the PeerWatch before any collective, or from the short process-group
    timeout of the collective itself."""
    import datetime
    import sys
    import time
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from riallm_b200.ep import ExpertParallelMoE, PeerWatch, RankFailureError
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=20))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    watch = PeerWatch(store, rank, world, timeout_s=2.0) if use_watch else None

    def ops(xt, e_begin, e_local):
        return torch.zeros(xt.shape, dtype=torch.float32)

    blk = ExpertParallelMoE({}, E, K, ops=ops, watch=watch)
    x = torch.zeros(T_LOCAL, H, dtype=torch.bfloat16)
    blk(x)
    if rank == 1:
        # Leave without tearing down the group: a process that died.
        os._exit(0)
    t0 = time.time()
    try:
        blk(x)
        msg = "no error"
    except RankFailureError as exc:
        msg = f"RankFailureError ranks={list(exc.ranks)} after {time.time() - t0:.1f}s"
    with open(os.path.join(result_dir, "rank0.txt"), "w") as f:
        f.write(msg)
    os._exit(0)


@pytest.mark.parametrize("use_watch", [True, False])
def test_rank_that_leaves_is_reported(tmp_path, use_watch):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_leaver, args=(r, 2, port, str(tmp_path), use_watch)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
        assert not p.is_alive()
    msg = open(tmp_path / "rank0.txt").read()
    assert msg.startswith("RankFailureError"), msg
    if use_watch:
        assert "ranks=[1]" in msg, msg


def test_exchange_plan_places_rows_expert_major(rb):
    """riallm_ep_exchange_plan (host-only): rows received from every rank
    land expert-major, ranks ascending inside an expert."""
    import ctypes
    L = rb.lib()
    W, EL = 3, 2
    rc = np.array([[2, 0], [1, 3], [0, 4]], np.int32)  # [source rank][local expert]
    cnt = np.zeros(EL, np.int32)
    off = np.zeros(EL + 1, np.int32)
    pos = np.zeros((W, EL), np.int32)
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    assert L.riallm_ep_exchange_plan(W, EL, p(rc), p(cnt), p(off), p(pos)) == 0
    assert cnt.tolist() == [3, 7] and off.tolist() == [0, 3, 10]
    assert pos.tolist() == [[0, 3], [2, 3], [3, 6]]
    assert L.riallm_ep_exchange_plan(0, EL, p(rc), p(cnt), p(off), p(pos)) != 0


def test_all_to_all_handle_argument_checks():
    """The all-to-all handle refuses an unknown transport, and the
    peer-memory transport without a token capacity, before it touches the
    process group or the GPU."""
    from riallm_b200 import ConfigError
    from riallm_b200.ep import ExpertParallelA2A
    with pytest.raises(ConfigError, match="transport"):
        ExpertParallelA2A({}, 8, 2, transport="shm")
    with pytest.raises(ConfigError, match="max_tokens"):
        ExpertParallelA2A({}, 8, 2, transport="peer", max_tokens=0)
