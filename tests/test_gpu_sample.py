"""nanoGPT sampling module ("generate") through the C ABI against the oracle.

generate-token (examples/nanogpt/model.shf:116-125) repeated with the window
update and key threading of examples/nanogpt/sample.shf:28-45. Every step is
checked on its own: the device's last-position logits against the oracle
forward of the device's own window, then the oracle sampler, fed those same
logits and the threaded key, must pick the device's token. The keys do not
depend on the logits, so the final keys must match exactly; the final window
must be the prompt window with the tokens rolled in.
"""
import numpy as np
import pytest

from oracle import dtype as odt
from oracle import models, prng, sampling
from tests.parity import TOL_BF16, TOL_F32, assert_close

pytestmark = pytest.mark.gpu

BF16 = 0x22000010
F32 = 0x21000020
CFG = models.GPTConfig(n_layer=2, n_head=2, n_embd=128, block_size=64, vocab_size=65, batch=3, seq=64)


def _prompt(cfg, seed=5):
    """encode-prompt (sample.shf:17-23): a zero window with the prompt ids
    rolled in; each sequence gets a prompt of a different length."""
    rng = np.random.default_rng(seed)
    ids = np.zeros((cfg.batch, cfg.block_size), np.float32)
    for b in range(cfg.batch):
        n = 1 + 7 * b
        ids[b, -n:] = rng.integers(0, cfg.vocab_size, n)
    return ids


def _generate(s, elem, leaves, ids, keys):
    ins = [s.upload(a, elem) for a in leaves] + [s.upload(ids, F32), s.upload(keys, F32)]
    return [o.to_host() for o in s.call("gpt.generate", ins)]


def _session(kind, n_new, top_k, temp, cfg=CFG):
    from sheaf_b200.runtime import Session

    s = Session(0)
    elem = BF16 if kind == "bf16" else F32
    s.create_gpt_sampler("gpt", n_layer=cfg.n_layer, n_head=cfg.n_head, n_embd=cfg.n_embd,
                         block_size=cfg.block_size, vocab_size=cfg.vocab_size, batch=cfg.batch, n_new=n_new,
                         top_k=top_k, temperature=temp, elem=elem)
    return s, elem


@pytest.mark.parametrize("kind,top_k,temp", [("f32", 200, 0.8), ("bf16", 200, 0.8), ("bf16", 5, 1.0),
                                             ("f32", 1, 1.0)])
def test_generate_matches_oracle(kind, top_k, temp, cuda):
    n_new = 6
    s, elem = _session(kind, n_new, top_k, temp)
    p, _, _ = models.gpt_inputs(CFG)
    bf = kind == "bf16"
    p = [odt.round_bf16(a) if bf else a.astype(np.float32) for a in p]
    ids0 = _prompt(CFG)
    keys0 = np.stack([prng.random_key(1337 + b) for b in range(CFG.batch)]).astype(np.float32)
    tokens, ids1, keys1, step_logits = _generate(s, elem, p, ids0, keys0)
    assert tokens.shape == (CFG.batch, n_new) and step_logits.shape == (n_new, CFG.batch, CFG.vocab_size)
    tol = TOL_BF16 if bf else TOL_F32
    k = min(top_k, CFG.vocab_size)
    near_ties = 0
    for b in range(CFG.batch):
        window, key = ids0[b].copy(), keys0[b].copy()
        for step in range(n_new):
            ref = models.gpt_forward_logits(p, window[None], CFG)[0, -1]
            assert_close(step_logits[step, b], ref, tol, f"seq {b} step {step} logits")
            tok, key, margin = sampling.generate_token(step_logits[step, b], key, k, temp)
            got = int(tokens[b, step])
            assert 0 <= got < CFG.vocab_size and float(tokens[b, step]) == got
            if margin < 1e-6:
                near_ties += 1  # u within float32 rounding of a cumsum edge
            else:
                assert got == tok, (b, step, got, tok, margin)
            if top_k == 1:
                assert got == int(np.argmax(step_logits[step, b]))
            window = sampling.slide_window(window, got)
        assert np.array_equal(ids1[b], window), b
        assert np.array_equal(keys1[b], key), b
    assert near_ties <= 1


def test_generate_is_deterministic_across_eager_and_graph(cuda):
    """The first token runs eagerly, the second is captured, the rest replay
    the graph; a second call replays from the start. Both calls agree bitwise
    and a call chained on the first's outputs continues the stream."""
    s, elem = _session("bf16", 5, 200, 0.8)
    p, _, _ = models.gpt_inputs(CFG)
    p = [odt.round_bf16(a) for a in p]
    ids0 = _prompt(CFG, seed=9)
    keys0 = np.stack([prng.random_key(b) for b in range(CFG.batch)]).astype(np.float32)
    r1 = _generate(s, elem, p, ids0, keys0)
    r2 = _generate(s, elem, p, ids0, keys0)
    for a, b in zip(r1, r2):
        assert np.array_equal(a, b)
    # the same 10 tokens from two chained calls of 5 as from one call of 10
    r3 = _generate(s, elem, p, r1[1], r1[2])
    s10, elem10 = _session("bf16", 10, 200, 0.8)
    r10 = _generate(s10, elem10, p, ids0, keys0)
    assert np.array_equal(r10[0], np.concatenate([r1[0], r3[0]], axis=1))
    assert np.array_equal(r10[1], r3[1]) and np.array_equal(r10[2], r3[2])


def test_generate_rejects_bad_inputs(cuda):
    import ctypes as C

    from sheaf_b200 import _lib
    from sheaf_b200.runtime import SheafB200Error, Session, _check, lib

    s, elem = _session("bf16", 2, 200, 0.8)
    p, _, _ = models.gpt_inputs(CFG)
    ids0 = _prompt(CFG)
    bad_keys = np.zeros((CFG.batch, 2), np.float32)
    with pytest.raises(SheafB200Error) as e:
        _generate(s, elem, p, ids0, bad_keys)
    assert e.value.code == 3
    s2 = Session(0)
    c = CFG
    gc = _lib.GptConfig(c.n_layer, c.n_head, c.n_embd, c.block_size, c.vocab_size, c.batch, c.block_size // 2, elem)
    sc = _lib.SamplerConfig(2, 200, 0.8)
    with pytest.raises(SheafB200Error):  # window shorter than block_size
        _check(lib().sb_module_create_gpt_sampler(s2._h, b"g", C.byref(gc), C.byref(sc)))
    with pytest.raises(SheafB200Error):
        s2.create_gpt_sampler("g", n_layer=1, n_head=2, n_embd=128, block_size=64, vocab_size=65, batch=1,
                              n_new=2, temperature=0.0)


@pytest.mark.parametrize("V,top_k", [(5000, 200), (50304, 200), (50304, 50304)])
def test_generate_large_vocabulary(V, top_k, cuda):
    """Vocabularies beyond one CTA's shared-memory sort (GPT-2's 50304): the
    logits are sorted per sequence with the chunked merge sort and the
    softmax / cumulative sum / choice run as block-wide scans. Per step: the
    logits against the oracle forward; with top_k = 200 the oracle sampler
    must pick the device's token (one near tie allowed); over the whole
    vocabulary the 50304 cumulative probabilities are ~2e-5 apart, closer than
    a float32 sum of them is accurate, so there the device's pick must be a
    valid draw for u under the exact cumulative sums within 1e-4."""
    cfg = models.GPTConfig(n_layer=1, n_head=2, n_embd=128, block_size=64, vocab_size=V, batch=2, seq=64)
    n_new, temp = 3, 0.8
    s, elem = _session("bf16", n_new, top_k, temp, cfg)
    p, _, _ = models.gpt_inputs(cfg)
    p = [odt.round_bf16(a) for a in p]
    ids0 = _prompt(cfg)
    keys0 = np.stack([prng.random_key(77 + b) for b in range(cfg.batch)]).astype(np.float32)
    tokens, ids1, keys1, step_logits = _generate(s, elem, p, ids0, keys0)
    near_ties = 0
    for b in range(cfg.batch):
        window, key = ids0[b].copy(), keys0[b].copy()
        for step in range(n_new):
            ref = models.gpt_forward_logits(p, window[None], cfg)[0, -1]
            assert_close(step_logits[step, b], ref, TOL_BF16, f"seq {b} step {step} logits")
            got = int(tokens[b, step])
            assert 0 <= got < V and float(tokens[b, step]) == got
            x = (np.asarray(step_logits[step, b], np.float32) / np.float32(temp)).astype(np.float32)
            vals, idx = sampling.top_k(x, min(top_k, V))
            new_key, subkey = prng.random_split(key, 2)
            if top_k < V:
                tok, _, margin = sampling.generate_token(step_logits[step, b], key, top_k, temp)
                if margin < 1e-6:
                    near_ties += 1
                else:
                    assert got == tok, (b, step, got, tok, margin)
            else:
                e = np.exp(vals.astype(np.float64) - vals.max())
                c = np.cumsum(e / e.sum())
                u = float(prng.random_uniform(subkey, ()))
                pos = int(np.nonzero(idx == got)[0][0])
                lo = c[pos - 1] if pos > 0 else 0.0
                assert lo <= u + 1e-4 and (c[pos] > u - 1e-4 or pos == len(c) - 1), (b, step, pos, lo, c[pos], u)
            key = new_key
            window = sampling.slide_window(window, got)
        assert np.array_equal(ids1[b], window), b
        assert np.array_equal(keys1[b], key), b
    assert near_ties <= 1
