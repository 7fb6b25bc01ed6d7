"""The sampling oracle (test-only restatement of generate-token,
examples/nanogpt/model.shf:116-125) against the reference's two forms of
choice and the properties its pieces must have. The PRNG underneath is pinned
by the Threefry known answers in test_oracle_goldens.py."""
import numpy as np

from oracle import prng, sampling

F = np.float32


def _interpreter_choice(subkey, probs):
    """sheaf/src/interpreter/builtins/random.rs:122-148: the first i with
    u < cumsum, else the last index."""
    u = F(prng.random_uniform(subkey, ()))
    c = F(0.0)
    for i, p in enumerate(np.asarray(probs, F)):
        c = F(c + p)
        if u < c:
            return i
    return len(probs) - 1


def test_lowered_choice_matches_interpreter_choice():
    """random_ops.rs:164-180 (count of cumsum > u) and the interpreter's scan
    agree for every key and distribution, zero-probability entries included."""
    rng = np.random.default_rng(0)
    for seed in range(300):
        key = prng.random_key(seed)
        k = int(rng.integers(1, 70))
        p = rng.random(k).astype(F)
        p[rng.random(k) < 0.2] = 0.0
        p = (p / max(p.sum(), F(1e-30))).astype(F)
        got, _ = sampling.choice_index(key, p)
        assert got == _interpreter_choice(key, p), seed


def test_choice_never_picks_a_zero_probability_entry():
    """The (choice key 4 :p [0.0 0.25 0.25 0.5]) case of prng_tests.rs."""
    p = np.array([0.0, 0.25, 0.25, 0.5], F)
    seen = set()
    for seed in [0, 42, 16777217, 4294967295, -1] + list(range(1, 200)):
        i, _ = sampling.choice_index(prng.random_key(seed), p)
        assert i != 0
        seen.add(i)
    assert seen == {1, 2, 3}


def test_top_k_is_stable_and_descending():
    x = np.array([1.0, 3.0, 3.0, -2.0, 3.0, 0.5], F)
    v, i = sampling.top_k(x, 4)
    assert list(i) == [1, 2, 4, 0] and list(v) == [3.0, 3.0, 3.0, 1.0]


def test_softmax_and_temperature():
    v = np.array([2.0, 1.0, -1.0], F)
    p = sampling.softmax_f32(v)
    assert p.dtype == F and abs(float(p.sum()) - 1.0) < 1e-6 and p[0] > p[1] > p[2]
    # top_k = 1 is greedy whatever the key
    logits = np.random.default_rng(1).standard_normal(65).astype(F)
    for seed in range(20):
        tok, _, _ = sampling.generate_token(logits, prng.random_key(seed), 1, 0.8)
        assert tok == int(np.argmax(logits))


def test_generate_token_threads_the_key():
    """[new-key subkey] = random-split(key): the returned key is child 0 and
    the draw uses child 1, whatever the logits."""
    key = prng.random_key(7)
    a, b = prng.random_split(key, 2)
    tok, new_key, _ = sampling.generate_token(np.zeros(65, F), key, 200, 1.0)
    assert np.array_equal(new_key, a)
    u = float(prng.random_uniform(b, ()))
    assert tok == min(int(u * 65), 64)  # uniform probabilities: index = floor(u * k) up to rounding
    assert np.array_equal(sampling.slide_window(np.arange(4, dtype=F), 9), np.array([1, 2, 3, 9], F))
