"""GPU parity of the router and bucketing (src/model.rs:762-789): top-k
indices, renormalised weights, per-expert counts, offsets and permutation
order bit-exact against the oracle."""
import numpy as np
import pytest
import torch

from conftest import load_golden

pytestmark = pytest.mark.gpu


def test_router_golden_bit_exact(rb):
    g = load_golden("router.npz")
    for tag in [k[2:] for k in g if k.startswith("x_")]:
        E = int(tag.split("_E")[1].split("_")[0])
        k = int(tag.split("_k")[1])
        x = torch.from_numpy(g[f"x_{tag}"].view(np.int16)).cuda().view(torch.bfloat16)
        wg = torch.from_numpy(g[f"wg_{tag}"]).cuda()
        idx, w, counts, offsets, perm = rb.route(wg, x, k, E)
        torch.cuda.synchronize()
        assert np.array_equal(idx.cpu().numpy(), g[f"idx_{tag}"]), tag
        assert np.array_equal(w.cpu().numpy().view(np.uint32), g[f"w_{tag}"].view(np.uint32)), tag
        assert np.array_equal(counts.cpu().numpy(), g[f"counts_{tag}"]), tag
        assert np.array_equal(offsets.cpu().numpy(), g[f"offsets_{tag}"]), tag
        assert np.array_equal(perm.cpu().numpy(), g[f"perm_{tag}"]), tag


@pytest.mark.parametrize("T,H,E,k,qt,bf16", [
    (64, 4096, 8, 2, 1, True),      # Mixtral-8x7B router, NF4-quantized (32768 >= 4096)
    (1, 4096, 8, 2, 1, True),
    (333, 2048, 128, 8, 2, True),   # fine-grained 128-expert top-8, 8-bit router
    (4096, 1024, 8, 2, 1, True),
    (50, 512, 16, 4, 1, False),     # float32 activations
    (200, 2048, 256, 16, 1, True),  # widest supported: 256 experts, top-16
    (7, 1024, 8, 2, 0, True),       # float32 router weight
    # One token per CTA with a float32 weight: eight chunks loaded ahead,
    # several experts per warp, a partial last group of chunks.
    (64, 2048, 128, 8, 0, True),
    (45, 1536, 24, 4, 0, False),
    # Prefill sizes: 8 (hidden <= 3072) or 4 tokens per router CTA, a ragged
    # last tile, and above 16384 pairs the multi-CTA pair sort.
    (1001, 2048, 128, 8, 1, True),
    (2051, 2048, 128, 8, 2, True),  # 16408 pairs: multi-CTA sort, ragged tile
    (517, 6144, 8, 2, 1, True),     # 4 tokens per CTA (hidden 6144)
    (3000, 1024, 256, 16, 0, True),  # 48000 pairs, float32 router, 256 experts
    (700, 512, 16, 4, 1, False),    # float32 activations, tiled
])
def test_router_random_bit_exact(rb, oracle_lib, T, H, E, k, qt, bf16):
    O = oracle_lib
    rng = np.random.default_rng(T * 7 + E)
    wg = rng.normal(0, 0.02, (E, H)).astype(np.float32)
    x = O.synthetic_x(T, H, T + 1, bf16=bf16)
    if qt == 0:
        _, _, idx_ref, w_ref = O.router(x, wg, k)
        dev = torch.from_numpy(wg).cuda()
    else:
        qwg = O.quantize(wg, qt)
        _, _, idx_ref, w_ref = O.router(x, O.dequantize(qwg).reshape(E, H), k)
        dev = rb.QuantizedTensor(torch.from_numpy(qwg.data).cuda(), (E, H), rb.CompressionType(qt),
                                 torch.from_numpy(qwg.scales).cuda(), torch.from_numpy(qwg.zero_points).cuda(),
                                 qwg.block_size)
    counts_ref, offsets_ref, perm_ref = O.bucket(idx_ref, E)
    xt = torch.from_numpy(x.view(np.int16)).cuda().view(torch.bfloat16) if bf16 else torch.from_numpy(x).cuda()
    idx, w, counts, offsets, perm = rb.route(dev, xt, k, E)
    assert np.array_equal(idx.cpu().numpy(), idx_ref)
    assert np.array_equal(w.cpu().numpy().view(np.uint32), w_ref.view(np.uint32))
    assert np.array_equal(counts.cpu().numpy(), counts_ref)
    assert np.array_equal(offsets.cpu().numpy(), offsets_ref)
    assert np.array_equal(perm.cpu().numpy(), perm_ref)


def test_router_ties_lower_index(rb):
    x = torch.ones(3, 256, device="cuda", dtype=torch.bfloat16)
    wg = torch.zeros(8, 256, device="cuda")
    idx, w, *_ = rb.route(wg, x, 3, 8)
    assert idx.cpu().tolist() == [[0, 1, 2]] * 3


def test_router_back_to_back_calls(rb, oracle_lib):
    """The pair sort runs in whichever CTA finishes last, found through a
    device counter that each call leaves at zero: consecutive calls with
    different token counts must each sort all of their own pairs."""
    O = oracle_lib
    rng = np.random.default_rng(5)
    E, H, k = 8, 1024, 2
    wg = rng.normal(0, 0.02, (E, H)).astype(np.float32)
    for T in (5, 300, 1, 64, 300):
        x = O.synthetic_x(T, H, T, bf16=True)
        _, _, idx_ref, _ = O.router(x, wg, k)
        counts_ref, offsets_ref, perm_ref = O.bucket(idx_ref, E)
        xt = torch.from_numpy(x.view(np.int16)).cuda().view(torch.bfloat16)
        idx, w, counts, offsets, perm = rb.route(torch.from_numpy(wg).cuda(), xt, k, E)
        assert np.array_equal(idx.cpu().numpy(), idx_ref), T
        assert np.array_equal(counts.cpu().numpy(), counts_ref), T
        assert np.array_equal(offsets.cpu().numpy(), offsets_ref), T
        assert np.array_equal(perm.cpu().numpy(), perm_ref), T
