"""End-to-end greedy decoding of a small Mixtral-style decoder whose MoE
blocks run on the GPU path, against the oracle's numpy decoder fed the same
tokens.

Checks per step: the last-position logits within 2e-2 (max |gpu - ref| /
max |ref|), and the greedy token equal to the oracle's argmax unless the
two candidates' oracle logits lie within that tolerance of each other.
"""
import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu

TOL = 2e-2


def _oracle_weights(O, qw):
    out, shapes = {}, {}
    for k, v in qw.items():
        if hasattr(v, "scales"):
            numel = int(np.prod(v.shape))
            out[k] = O.QTensor(int(v.qtype), v.data.cpu().numpy(), v.scales.cpu().numpy(),
                               v.zero_points.cpu().numpy(), numel, v.block_size)
            shapes[k] = tuple(v.shape)
        else:
            out[k] = v.float().cpu().numpy()
    return out, shapes


def test_greedy_decode_matches_oracle(rb, oracle_lib):
    from oracle.decoder_ref import DecoderRef
    from riallm_b200 import decoder as D
    cfg = D.DecoderConfig()
    qw = D.quantize_weights(D.synthetic_weights(cfg, seed=0))
    model = D.TinyDecoder(cfg, qw)
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, cfg.vocab, (64,), generator=g)
    new = 16
    toks, logits = model.generate(prompt.cuda(), new, keep_logits=True)
    logits = logits.cpu().numpy()
    assert len(toks) == new and logits.shape == (new, cfg.vocab)

    ow, shapes = _oracle_weights(oracle_lib, qw)
    ref = DecoderRef(cfg, ow, shapes)
    feed, pos, flips = prompt.numpy(), 0, 0
    for s in range(new):
        r = ref.forward(feed, pos, last_only=True)[0]
        pos += len(feed)
        e = rel_err(logits[s], r)
        assert e < TOL, f"step {s}: logits rel err {e}"
        want = int(np.argmax(r))
        if toks[s] != want:
            flips += 1
            gap = (r[want] - r[toks[s]]) / np.abs(r).max()
            assert gap < TOL, f"step {s}: token {toks[s]} vs oracle {want}, gap {gap}"
        feed = np.array([toks[s]])
    assert flips <= 2
