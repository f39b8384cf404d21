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


class _OneRank:
    """The one call of torch.distributed that ep_compare makes, for a single
    rank (the maximum over one rank is the value itself)."""

    class ReduceOp:
        MAX = "max"

    @staticmethod
    def all_reduce(t, op=None):
        return t


def test_ep_compare_allows_one_bf16_rounding_step_only():
    """The expert-parallel check passes identical outputs and outputs that
    differ by one bf16 rounding step of an element; two steps on a large
    element fail it."""
    g = torch.Generator().manual_seed(9)
    ref = (torch.randn(16, 64, generator=g) * 3).to(torch.bfloat16)
    assert bench.ep_compare(torch, _OneRank, ref.clone(), ref)["passed"]
    bits = ref.view(torch.int16).clone()
    i = int(ref.float().abs().argmax())
    one = bits.clone()
    one.view(-1)[i] += 1  # the next bf16 value of the largest element
    r1 = bench.ep_compare(torch, _OneRank, one.view(torch.bfloat16), ref)
    assert r1["passed"] and r1["max_ulps"] == 1.0 and r1["elements_beyond_bound"] == 0
    two = bits.clone()
    two.view(-1)[i] += 2
    r2 = bench.ep_compare(torch, _OneRank, two.view(torch.bfloat16), ref)
    assert not r2["passed"] and r2["elements_beyond_bound"] == 1
