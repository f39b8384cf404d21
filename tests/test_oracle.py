"""CPU tests of the oracle: the C restatement against the committed golden
fixtures, against the independent numpy mirror, and against answers derived
by hand from the reference source on the reference's own test inputs
(tests/integration_test.rs:124-148 in the riallm crate)."""
import math

import numpy as np
import pytest

from conftest import load_golden


def bits(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


def test_golden_quant_reproduces(oracle_lib):
    O = oracle_lib
    g = load_golden("quant.npz")
    for key in [k for k in g if k.startswith("v_")]:
        n = int(key[2:])
        v = g[key]
        for name, qt in (("nf4", O.FOUR_BIT), ("int8", O.EIGHT_BIT)):
            t = O.quantize(v, qt)
            assert np.array_equal(t.data, g[f"{name}_data_{n}"]), (name, n)
            assert np.array_equal(bits(t.scales), bits(g[f"{name}_scales_{n}"])), (name, n)
            assert np.array_equal(bits(t.zero_points), bits(g[f"{name}_zeros_{n}"])), (name, n)
            assert np.array_equal(bits(O.dequantize(t)), bits(g[f"{name}_deq_{n}"])), (name, n)


@pytest.mark.parametrize("n", [1, 2, 3, 63, 64, 65, 127, 128, 129, 257, 4096, 4097, 12345])
def test_numpy_mirror_agrees(oracle_lib, n):
    O = oracle_lib
    rng = np.random.default_rng(n)
    v = rng.normal(0, 0.3, n).astype(np.float32)
    t = O.quantize(v, O.FOUR_BIT)
    d, s, z = O.np_quantize_nf4(v)
    assert np.array_equal(d, t.data)
    assert np.array_equal(bits(s), bits(t.scales))
    assert np.array_equal(bits(z), bits(t.zero_points))
    deq = O.dequantize(t)
    assert deq.size == n
    assert np.array_equal(bits(deq), bits(O.np_dequantize_nf4(t.data, t.scales, t.zero_points, n)))
    assert np.array_equal(bits(deq), bits(O.tensor_span(t, 0, n)))
    t8 = O.quantize(v, O.EIGHT_BIT)
    d8, s8, z8 = O.np_quantize_int8(v)
    assert np.array_equal(d8, t8.data)
    assert np.array_equal(bits(s8), bits(t8.scales)) and np.array_equal(bits(z8), bits(t8.zero_points))
    assert np.array_equal(bits(O.dequantize(t8)), bits(O.np_dequantize_int8(t8.data, t8.scales, t8.zero_points)))


def test_pin_reference_quantize_8bit_input(oracle_lib):
    """tests/integration_test.rs:125-135: (0..256)/255 as [16,16]. Two
    128-blocks; the reference's formula round((v-min)/((max-min)/255)) gives
    round(255 j / 127) in both blocks (never a .5 tie: 127 is odd)."""
    O = oracle_lib
    data = (np.arange(256, dtype=np.float32) / np.float32(255.0)).astype(np.float32)
    t = O.quantize(data, O.EIGHT_BIT)
    j = np.arange(128)
    expect = np.floor(255.0 * j / 127.0 + 0.5).astype(np.uint8)
    assert t.scales.size == 2 and t.zero_points.size == 2
    assert np.array_equal(t.data[:128], expect) and np.array_equal(t.data[128:], expect)
    assert t.zero_points[0] == 0.0 and t.zero_points[1] == np.float32(128) / np.float32(255)
    assert abs(t.scales[0] - (127 / 255) / 255) < 1e-9
    # dequantize_8bit is (q - zero) * scale (src/quantization.rs:91), not q*scale + zero
    deq = O.dequantize(t)
    q, s, z = np.float32(t.data[200]), t.scales[1], t.zero_points[1]
    assert deq[200] == np.float32(np.float32(q - z) * s)


def test_pin_reference_quantize_4bit_input(oracle_lib):
    """tests/integration_test.rs:138-147: x/128 - 0.5 for x in 0..128 as
    [8,16]. Codes by hand from the table at src/quantization.rs:127-130:
    -0.5 -> 2 (-0.525), -0.25 -> 4 (-0.275), -0.125 -> 6 (-0.085), 0 -> 8,
    0.4921875 -> 14 (0.525)."""
    O = oracle_lib
    v = (np.arange(128, dtype=np.float32) / np.float32(128.0) - np.float32(0.5)).astype(np.float32)
    t = O.quantize(v, O.FOUR_BIT)
    code = lambda e: (t.data[e >> 1] >> 4) & 15 if e & 1 else t.data[e >> 1] & 15
    assert [code(e) for e in (0, 1, 32, 48, 60, 62, 63, 64, 127)] == [2, 2, 4, 6, 7, 7, 7, 8, 14]
    assert t.data[0] == 0x22
    assert t.scales.tolist() == [0.5, 0.4921875]
    assert t.zero_points.tolist() == [-0.25390625, 0.24609375]
    deq = O.dequantize(t)
    f = np.float32
    assert deq[0] == f(f(2 - f(-0.25390625)) * f(0.5))
    # element 63 (last of block 0) reads block 1's scale and zero
    assert deq[63] == f(f(7 - f(0.24609375)) * f(0.4921875))
    # the tensor's last element reads past the scale vector: defaults 1.0 / 0.0
    assert deq[127] == 14.0
    assert deq[62] == f(f(7 - f(-0.25390625)) * f(0.5))


def test_nf4_odd_tail_and_empty(oracle_lib):
    O = oracle_lib
    v = np.array([0.3, -0.2, 0.5], np.float32)
    t = O.quantize(v, O.FOUR_BIT)
    assert t.data.size == 2 and t.scales.size == 1
    # second byte: low = code(0.5) = 14 (0.525), high pad = code(0.0) = 8
    assert t.data[1] == (8 << 4) | 14
    assert O.dequantize(t).size == 3


def test_int8_constant_block_is_nan_then_zero(oracle_lib):
    """A constant block has scale 0: (v-min)/0 = NaN, and Rust's `as u8`
    maps NaN to 0 (src/quantization.rs:232)."""
    O = oracle_lib
    t = O.quantize(np.full(130, 0.25, np.float32), O.EIGHT_BIT)
    assert (t.data == 0).all() and t.scales[0] == 0.0


def test_own_expf_accuracy(oracle_lib):
    O = oracle_lib
    xs = np.concatenate([np.linspace(-87, 0, 20001), [-1e-8, -0.0, 0.0]]).astype(np.float32)
    worst = 0.0
    for x in xs:
        ref = math.exp(float(x))
        worst = max(worst, abs(O.expf(float(x)) - ref) / ref)
    assert worst < 1.5e-7  # about 1 ulp
    assert O.expf(-100.0) == 0.0


@pytest.mark.parametrize("T,H,E,k,seed", [(512, 4096, 8, 2, 1), (512, 2048, 128, 8, 2)])
def test_router_softmax_matches_float64(oracle_lib, T, H, E, k, seed):
    """How far the router's own softmax (own exp, sequential sum in expert
    order, IEEE division) moves from an exact softmax of the same float32
    logits: a few float32 ulps in the probabilities, fewer in the
    renormalised routing weights, and the same top-k set wherever the k-th
    and (k+1)-th probabilities differ by more than that. (candle's softmax
    and the order of its logit GEMM are not observable here.)"""
    O = oracle_lib
    rng = np.random.default_rng(seed)
    wg = rng.normal(0, 0.02, (E, H)).astype(np.float32)
    x = O.synthetic_x(T, H, seed + 10, bf16=True)
    logits, probs, idx, w = O.router(x, wg, k)
    l64 = logits.astype(np.float64)
    p64 = np.exp(l64 - l64.max(axis=1, keepdims=True))
    p64 /= p64.sum(axis=1, keepdims=True)
    assert (np.abs(probs - p64) / p64).max() < 2e-6
    w64 = np.take_along_axis(p64, idx.astype(np.int64), axis=1)
    w64 /= w64.sum(axis=1, keepdims=True)
    assert (np.abs(w - w64) / w64).max() < 1e-6
    top = -np.sort(-p64, axis=1)
    gap = (top[:, k - 1] - top[:, k]) / top[:, k - 1]
    exact = np.sort(np.argsort(-p64, axis=1, kind="stable")[:, :k], axis=1)
    clear = gap > 4e-6
    assert clear.mean() > 0.99
    assert np.array_equal(exact[clear], np.sort(idx, axis=1)[clear])


def test_router_golden_and_stability(oracle_lib):
    O = oracle_lib
    g = load_golden("router.npz")
    for tag in [k[2:] for k in g if k.startswith("x_")]:
        k = int(tag.split("_k")[1])
        E = int(tag.split("_E")[1].split("_")[0])
        logits, probs, idx, w = O.router(g[f"x_{tag}"], g[f"wg_{tag}"], k)
        assert np.array_equal(bits(logits), bits(g[f"logits_{tag}"]))
        assert np.array_equal(idx, g[f"idx_{tag}"])
        assert np.array_equal(bits(w), bits(g[f"w_{tag}"]))
        counts, offsets, perm = O.bucket(idx, E)
        assert np.array_equal(counts, g[f"counts_{tag}"]) and np.array_equal(perm, g[f"perm_{tag}"])
        # top-k is the stable descending order of the probabilities
        for t in range(idx.shape[0]):
            order = sorted(range(E), key=lambda e: (-probs[t, e], e))[:k]
            assert list(idx[t]) == order


def test_router_ties_go_to_lower_index(oracle_lib):
    O = oracle_lib
    x = np.ones((1, 256), np.float32)
    wg = np.zeros((8, 256), np.float32)  # all logits equal
    _, _, idx, w = O.router(x, wg, 3)
    assert idx.tolist() == [[0, 1, 2]]
    assert np.allclose(w, 1 / 3)


def test_bucket_is_stable_counting_sort(oracle_lib):
    O = oracle_lib
    rng = np.random.default_rng(5)
    T, k, E = 50, 3, 7
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    counts, offsets, perm = O.bucket(idx, E)
    assert counts.sum() == T * k and offsets[-1] == T * k
    for e in range(E):
        seg = perm[offsets[e]:offsets[e + 1]]
        assert (idx.reshape(-1)[seg] == e).all()
        assert (np.diff(seg) > 0).all()  # token-ascending inside an expert


@pytest.mark.parametrize("name", ["moe_nf4_bf16", "moe_int8_bf16", "moe_nf4_f32",
                                  "moe_nf4_bf16_k4_e8", "moe_nf4_bf16_shared"])
def test_golden_moe_reproduces(oracle_lib, name):
    O = oracle_lib
    g = load_golden(name + ".npz")
    H, I, E, k, T, qt, bf16, shared_I = [int(v) for v in g["dims"]]

    def qtensor(n):
        qtype, bs, numel = [int(v) for v in g[f"{n}.qtype"]]
        return O.QTensor(qtype, g[f"{n}.data"], g[f"{n}.scales"], g[f"{n}.zeros"], numel, bs)

    w = O.MoeWeights(qtensor("gate"), qtensor("gate_up_proj"), qtensor("down_proj"))
    if shared_I:
        w.shared_gate_proj, w.shared_up_proj = qtensor("shared_gate_proj"), qtensor("shared_up_proj")
        w.shared_down_proj, w.shared_expert_gate = qtensor("shared_down_proj"), qtensor("shared_expert_gate")
        w.shared_intermediate = shared_I
    out, idx, tw, counts = O.moe_forward(w, g["x"], T, H, I, E, k)
    assert np.array_equal(idx, g["idx"]) and np.array_equal(counts, g["counts"])
    assert np.array_equal(bits(out), bits(g["out"]))


def test_moe_oracle_matches_float64_formula(oracle_lib):
    """The block equals sum_e w_e * down(silu(gate x) * up x) computed
    independently in float64 from the dequantized weights (fp32 mode)."""
    O = oracle_lib
    H, I, E, k, T = 256, 256, 4, 2, 3
    w, _ = O.synthetic_layer(H, I, E, O.FOUR_BIT, 11)
    x = O.synthetic_x(T, H, 12, bf16=False)
    out, idx, tw, _ = O.moe_forward(w, x, T, H, I, E, k)
    gu = O.dequantize(w.gate_up_proj).reshape(E, 2 * I, H).astype(np.float64)
    dn = O.dequantize(w.down_proj).reshape(E, H, I).astype(np.float64)
    ref = np.zeros((T, H))
    for t in range(T):
        for j in range(k):
            e = idx[t, j]
            p = gu[e] @ x[t].astype(np.float64)
            h = p[:I] / (1 + np.exp(-p[:I])) * p[I:]
            ref[t] += tw[t, j] * (dn[e] @ h)
    err = np.abs(out - ref).max() / np.abs(ref).max()
    assert err < 1e-5
