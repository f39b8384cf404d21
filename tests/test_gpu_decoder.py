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


def _check_against_oracle(O, cfg, qw, prompt, toks, logits):
    """Teacher-forces the oracle decoder with the GPU's tokens."""
    from oracle.decoder_ref import DecoderRef
    ow, shapes = _oracle_weights(O, qw)
    ref = DecoderRef(cfg, ow, shapes)
    feed, pos, flips = prompt, 0, 0
    for s in range(len(toks)):
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


@pytest.fixture(scope="module")
def tiny():
    from riallm_b200 import decoder as D
    cfg = D.DecoderConfig()
    return cfg, D.quantize_weights(D.synthetic_weights(cfg, seed=0))


def test_greedy_decode_matches_oracle(rb, oracle_lib, tiny):
    """64-token prompt (ids U[0, 32000), seed 1), 16 greedy tokens."""
    from riallm_b200 import decoder as D
    cfg, qw = tiny
    model = D.Decoder(cfg, qw)
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, cfg.vocab, (64,), generator=g)
    new = 16
    toks, logits = model.generate(prompt.cuda(), new, keep_logits=True)
    logits = logits.cpu().numpy()
    assert len(toks) == new and logits.shape == (new, cfg.vocab)
    _check_against_oracle(oracle_lib, cfg, qw, prompt.numpy(), toks, logits)
    # the eager path (no CUDA graph) gives the same tokens
    assert model.generate(prompt.cuda(), new, use_graph=False) == toks


def test_configured_tiny_model_greedy_tokens(rb, oracle_lib):
    """The tiny configuration exactly as specified: every weight N(0, 0.02)
    from seed 0 (experts included) and unit RMSNorm weights, NF4 MoE
    tensors; prompt of 64 ids U[0, 32000) seed 1, 16 greedy tokens.

    riallm's NF4 decode makes every expert weight about 7.5 x absmax, so the
    MoE blocks add a large, nearly rank-one term to the residual stream;
    the checks are the same as above, and every step's oracle margin
    between its best and second-best token is reported, so that a token
    that differs can be told from a near-tie of the oracle itself."""
    from oracle.decoder_ref import DecoderRef
    from riallm_b200 import decoder as D
    O = oracle_lib
    cfg = D.DecoderConfig()
    qw = D.quantize_weights(D.synthetic_weights(cfg, seed=0, expert_std=0.02, alt_norm=False))
    model = D.Decoder(cfg, qw)
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, cfg.vocab, (64,), generator=g)
    toks, logits = model.generate(prompt.cuda(), 16, keep_logits=True)
    logits = logits.cpu().numpy()
    ow, shapes = _oracle_weights(O, qw)
    ref = DecoderRef(cfg, ow, shapes)
    feed, pos, same, report = prompt.numpy(), 0, 0, []
    for s in range(16):
        r = ref.forward(feed, pos, last_only=True)[0]
        pos += len(feed)
        top2 = np.argsort(r)[-2:]
        margin = float((r[top2[1]] - r[top2[0]]) / np.abs(r).max())
        err = rel_err(logits[s], r)
        want = int(np.argmax(r))
        report.append((s, toks[s], want, err, margin))
        assert err < TOL, f"step {s}: logits rel err {err}"
        if toks[s] == want:
            same += 1
        else:
            gap = float((r[want] - r[toks[s]]) / np.abs(r).max())
            assert gap < TOL, f"step {s}: token {toks[s]} vs oracle {want}, oracle gap {gap}"
        feed = np.array([toks[s]])
    print("step gpu_token oracle_token logits_rel_err oracle_top2_margin")
    for row in report:
        print("%d %d %d %.3e %.3e" % row)
    print(f"identical greedy tokens: {same}/16")
    assert same == 16, "the configured model must reproduce the oracle's greedy tokens"
    model.close()


def test_batched_decode_matches_oracle(rb, oracle_lib, tiny):
    """Two sequences decoded together, each checked against the oracle."""
    from riallm_b200 import decoder as D
    cfg, qw = tiny
    model = D.Decoder(cfg, qw, max_batch=2, max_seq=128)
    g = torch.Generator().manual_seed(2)
    prompts = torch.randint(0, cfg.vocab, (2, 24), generator=g)
    toks, logits = model.generate(prompts.cuda(), 8, keep_logits=True)
    assert toks.shape == (2, 8) and logits.shape == (2, 8, cfg.vocab)
    for b in range(2):
        _check_against_oracle(oracle_lib, cfg, qw, prompts[b].numpy(), toks[b].tolist(), logits[b].cpu().numpy())
    with pytest.raises(rb.ConfigError, match="max_seq"):
        model.generate(prompts.cuda(), 200)


def test_forced_decode_and_expert_count(rb, tiny):
    """Teacher-forced decode steps (graph replays) advance the cache like
    eager steps: the logits of a following eager step match those of a model
    that decoded the same ids eagerly; the router probe reports, per layer,
    between top_k and E distinct experts."""
    from riallm_b200 import decoder as D
    cfg, qw = tiny
    g = torch.Generator().manual_seed(4)
    prompt = torch.randint(0, cfg.vocab, (2, 12), generator=g).cuda()
    forced = torch.randint(0, cfg.vocab, (5, 2, 1), generator=g).cuda()
    a, b = D.Decoder(cfg, qw, max_batch=2, max_seq=64), D.Decoder(cfg, qw, max_batch=2, max_seq=64)
    a.reset()
    a.forward(prompt)
    a.decode_forced(forced)
    b.reset()
    b.forward(prompt)
    for i in range(5):
        b.forward(forced[i])
    assert a.length == b.length == 17
    nxt = torch.randint(0, cfg.vocab, (2, 1), generator=g).cuda()
    la, lb = a.forward(nxt), b.forward(nxt)
    assert rel_err(la.cpu().numpy(), lb.cpu().numpy()) < 1e-2
    used = a.experts_per_layer(nxt)
    assert len(used) == cfg.layers and all(cfg.top_k <= u <= cfg.experts for u in used)
    a.close()
    b.close()
