"""Host-side pieces of bench.py that need no GPU: the fine-grained
configuration's Zipf expert-popularity bias and the warm-up floor."""
import math

import torch

import bench


def test_zipf_bias_is_a_seeded_permutation_of_the_law():
    b = bench.zipf_bias(torch, 128)
    assert b.shape == (128,) and b.dtype == torch.float32
    # exp(bias) is a probability distribution over the experts.
    assert abs(torch.exp(b.double()).sum().item() - 1.0) < 1e-6
    # Sorted, the biases follow ln(r^-1.1 / sum_r r^-1.1) for r = 1..128.
    z = sum(r ** -1.1 for r in range(1, 129))
    want = torch.tensor([math.log(r ** -1.1 / z) for r in range(1, 129)])
    got, _ = torch.sort(b.double(), descending=True)
    assert torch.allclose(got, want.double(), atol=1e-5)
    # The ranks come from a seeded permutation: same seed, same assignment.
    assert torch.equal(b, bench.zipf_bias(torch, 128))
    assert not torch.equal(b, bench.zipf_bias(torch, 128, seed=5))


def test_warmup_floor():
    assert bench.parse_args(["--warmup", "1"]).warmup == 3
    assert bench.parse_args(["--warmup", "7"]).warmup == 7
    args = bench.parse_args([])
    assert (args.gpus, args.tokens, args.impl) == (1, 64, "ours")
