"""Whole-program restatements: the MLP value-and-grad and the nanoGPT
value-and-grad (loss + 40 parameter gradients), composed from oracle.ops.

nanoGPT follows examples/nanogpt/model.shf:1-114 exactly:
  * pre-LN blocks, layer-norm without beta (layer-norm-nb, model.shf:11-14);
  * q/k/v from row slices of c_attn [3D, D], `x @ W^T` (model.shf:55-63);
  * scores / sqrt(Hd), `where(tril==1, s, -1e10)`, softmax (model.shf:66-68);
  * heads merged by swapaxes + reshape (model.shf:70), output projection;
  * MLP: gelu(x @ Wfc^T) @ Wproj^T (model.shf:74-80);
  * x = wte[idx] + wpe[0:T]; final layer-norm; logits = x @ lm_head^T
    (model.shf:97-113); loss = cross-entropy (lib/nn.shf:44-50).
Parameters are flattened in the order Sheaf passes pytree leaves to a
compiled module: dict keys sorted, lists in order
(sheaf/src/runtime/buffer_convert.rs:218-246).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import ops, prng

F32 = np.float32


@dataclass(frozen=True)
class GPTConfig:
    n_layer: int = 6
    n_head: int = 6
    n_embd: int = 384
    block_size: int = 256
    vocab_size: int = 65
    batch: int = 64
    seq: int = 256

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head


NANOGPT_CHAR = GPTConfig()
GPT2_SMALL = GPTConfig(n_layer=12, n_head=12, n_embd=768, block_size=1024, vocab_size=50304, batch=64, seq=1024)


def gpt_leaf_names(cfg: GPTConfig) -> list[str]:
    """Leaf order of the params pytree (sorted keys; `h` is a list)."""
    names = ["lm_head.weight"]
    for l in range(cfg.n_layer):
        for leaf in ("attn.c_attn.weight", "attn.c_proj.weight", "ln_1.weight", "ln_2.weight", "mlp.c_fc.weight",
                     "mlp.c_proj.weight"):
            names.append(f"transformer.h.{l}.{leaf}")
    names += ["transformer.ln_f.weight", "transformer.wpe.weight", "transformer.wte.weight"]
    return names


def gpt_leaf_shapes(cfg: GPTConfig) -> list[tuple[int, ...]]:
    D, V = cfg.n_embd, cfg.vocab_size
    shapes = [(V, D)]
    for _ in range(cfg.n_layer):
        shapes += [(3 * D, D), (D, D), (D,), (D,), (4 * D, D), (D, 4 * D)]
    shapes += [(D,), (cfg.block_size, D), (V, D)]
    return shapes


def init_gpt_params(key_limbs, cfg: GPTConfig) -> list[np.ndarray]:
    """init-gpt-params / init-block (examples/nanogpt/model.shf:17-43), as leaves."""
    D, V = cfg.n_embd, cfg.vocab_size
    k_wte, k_wpe, k_blocks, k_head = prng.random_split(key_limbs, 4)
    block_keys = prng.random_split(k_blocks, cfg.n_layer)
    s = F32(0.02)
    leaves = [prng.random_normal(k_head, (V, D)) * s]
    for bk in block_keys:
        k_attn, k_proj, k_fc, k_fc2 = prng.random_split(bk, 4)
        leaves += [prng.random_normal(k_attn, (3 * D, D)) * s, prng.random_normal(k_proj, (D, D)) * s,
                   np.ones(D, F32), np.ones(D, F32),
                   prng.random_normal(k_fc, (4 * D, D)) * s, prng.random_normal(k_fc2, (D, 4 * D)) * s]
    leaves += [np.ones(D, F32), prng.random_normal(k_wpe, (cfg.block_size, D)) * s,
               prng.random_normal(k_wte, (V, D)) * s]
    return [np.ascontiguousarray(x, dtype=F32) for x in leaves]


def gpt_inputs(cfg: GPTConfig, seed_params: int = 0, seed_x: int = 1, seed_y: int = 2):
    """Seeded synthetic workload: params from (random-key 0); token ids
    x, y = random-randint (random-key 1 / 2) [B, T] in [0, V) (f32 ids)."""
    params = init_gpt_params(prng.random_key(seed_params), cfg)
    x = prng.random_randint(prng.random_key(seed_x), (cfg.batch, cfg.seq), 0, cfg.vocab_size)
    y = prng.random_randint(prng.random_key(seed_y), (cfg.batch, cfg.seq), 0, cfg.vocab_size)
    return params, x, y


def gpt_value_and_grad(leaves, x_ids, y_ids, cfg: GPTConfig, dtype=np.float64, want_logits: bool = False):
    """Loss and gradients of `cross-entropy(gpt-forward(x, p), y)` w.r.t. every
    leaf, in leaf order. Computed in `dtype` (float64 by default)."""
    t = np.dtype(dtype).type
    P = [np.asarray(p, dtype=dtype) for p in leaves]
    L, H, D = cfg.n_layer, cfg.n_head, cfg.n_embd
    Hd = D // H
    B, T = np.asarray(x_ids).shape
    N = B * T
    head = P[0]
    blocks = [P[1 + 6 * l: 7 + 6 * l] for l in range(L)]
    ln_f, wpe, wte = P[1 + 6 * L], P[2 + 6 * L], P[3 + 6 * L]
    scale = t(np.sqrt(Hd))
    mask = np.tril(np.ones((T, T), dtype=bool))

    # forward
    x = ops.embedding(wte, x_ids) + wpe[:T][None]
    x = x.reshape(N, D)
    caches = []
    for (w_attn, w_proj, g1, g2, w_fc, w_fc2) in blocks:
        h1, c1 = ops.layer_norm_nb(x, g1)
        qkv = h1 @ w_attn.T
        q, k, v = (qkv[:, i * D:(i + 1) * D].reshape(B, T, H, Hd).transpose(0, 2, 1, 3) for i in range(3))
        s = (q @ np.swapaxes(k, -1, -2)) / scale
        s = np.where(mask, s, t(ops.MASK_FILL))
        p = ops.softmax(s)
        o = (p @ v).transpose(0, 2, 1, 3).reshape(N, D)
        x = x + o @ w_proj.T
        h2, c2 = ops.layer_norm_nb(x, g2)
        u = h2 @ w_fc.T
        gu = ops.gelu(u)
        x_in = x
        x = x + gu @ w_fc2.T
        caches.append((h1, c1, q, k, v, p, o, h2, c2, u, gu))
    hf, cf = ops.layer_norm_nb(x, ln_f)
    logits = hf @ head.T
    loss = ops.cross_entropy(logits, y_ids)

    # backward
    grads = [None] * len(P)
    dlogits = ops.cross_entropy_vjp(logits, y_ids)
    grads[0] = dlogits.T @ hf
    dhf = dlogits @ head
    dx, grads[1 + 6 * L] = ops.layer_norm_nb_vjp(cf, ln_f, dhf)
    for l in reversed(range(L)):
        w_attn, w_proj, g1, g2, w_fc, w_fc2 = blocks[l]
        h1, c1, q, k, v, p, o, h2, c2, u, gu = caches[l]
        base = 1 + 6 * l
        grads[base + 5] = dx.T @ gu
        dgu = dx @ w_fc2
        du = ops.gelu_vjp(u, dgu)
        grads[base + 4] = du.T @ h2
        dh2 = du @ w_fc
        dxl, grads[base + 3] = ops.layer_norm_nb_vjp(c2, g2, dh2)
        dx = dx + dxl
        grads[base + 1] = dx.T @ o
        do = (dx @ w_proj).reshape(B, T, H, Hd).transpose(0, 2, 1, 3)
        dv = np.swapaxes(p, -1, -2) @ do
        dp = do @ np.swapaxes(v, -1, -2)
        ds = ops.softmax_vjp(p, dp)
        ds = np.where(mask, ds, t(0.0)) / scale
        dq = ds @ k
        dk = np.swapaxes(ds, -1, -2) @ q
        dqkv = np.concatenate([z.transpose(0, 2, 1, 3).reshape(N, D) for z in (dq, dk, dv)], axis=1)
        grads[base + 0] = dqkv.T @ h1
        dh1 = dqkv @ w_attn
        dxl, grads[base + 2] = ops.layer_norm_nb_vjp(c1, g1, dh1)
        dx = dx + dxl
    dx3 = dx.reshape(B, T, D)
    grads[3 + 6 * L] = ops.embedding_vjp(wte.shape, x_ids, dx3, dtype)
    grads[2 + 6 * L] = ops.slice_rows_vjp(wpe.shape, 0, dx3.sum(axis=0))
    if want_logits:
        return loss, grads, logits
    return loss, grads


def gpt_forward_logits(leaves, x_ids, cfg: GPTConfig, dtype=np.float64):
    """Forward only (gpt-forward, model.shf:85-113): logits [B, T, V]."""
    t = np.dtype(dtype).type
    P = [np.asarray(p, dtype=dtype) for p in leaves]
    L, H, D = cfg.n_layer, cfg.n_head, cfg.n_embd
    Hd = D // H
    B, T = np.asarray(x_ids).shape
    N = B * T
    mask = np.tril(np.ones((T, T), dtype=bool))
    x = (ops.embedding(P[3 + 6 * L], x_ids) + P[2 + 6 * L][:T][None]).reshape(N, D)
    for l in range(L):
        w_attn, w_proj, g1, g2, w_fc, w_fc2 = P[1 + 6 * l: 7 + 6 * l]
        h1, _ = ops.layer_norm_nb(x, g1)
        qkv = h1 @ w_attn.T
        q, k, v = (qkv[:, i * D:(i + 1) * D].reshape(B, T, H, Hd).transpose(0, 2, 1, 3) for i in range(3))
        s = np.where(mask, (q @ np.swapaxes(k, -1, -2)) / t(np.sqrt(Hd)), t(ops.MASK_FILL))
        x = x + (ops.softmax(s) @ v).transpose(0, 2, 1, 3).reshape(N, D) @ w_proj.T
        h2, _ = ops.layer_norm_nb(x, g2)
        x = x + ops.gelu(h2 @ w_fc.T) @ w_fc2.T
    hf, _ = ops.layer_norm_nb(x, P[1 + 6 * L])
    return (hf @ P[0].T).reshape(B, T, -1)


# ---- MLP value-and-grad (x[64,784] -> 256 gelu -> 10, mse) -----------------

def mlp_inputs(batch: int = 64, d_in: int = 784, d_hidden: int = 256, d_out: int = 10):
    """Seeded workload: x = random-normal (random-key 0) [64, 784]; W1, W2 =
    xavier-uniform from random-split (random-key 0) 2 (lib/nn.shf:77-82);
    biases zero; y = one-hot(random-randint (random-key 1) [64] 0 10, 10).
    Leaves (sorted keys): l1.W, l1.b, l2.W, l2.b."""
    k1, k2 = prng.random_split(prng.random_key(0), 2)
    x = prng.random_normal(prng.random_key(0), (batch, d_in))
    w1 = prng.xavier_uniform(k1, (d_in, d_hidden))
    w2 = prng.xavier_uniform(k2, (d_hidden, d_out))
    labels = prng.random_randint(prng.random_key(1), (batch,), 0, d_out)
    y = ops.one_hot(labels, d_out, F32)
    return [w1, np.zeros(d_hidden, F32), w2, np.zeros(d_out, F32)], x, y


def mlp_value_and_grad(leaves, x, y, dtype=np.float64):
    """mse-loss(linear(gelu(linear(x, W1, b1)), W2, b2), y) (lib/nn.shf:106-117)."""
    w1, b1, w2, b2 = (np.asarray(p, dtype=dtype) for p in leaves)
    x = np.asarray(x, dtype=dtype)
    y = np.asarray(y, dtype=dtype)
    h = x @ w1 + b1
    a = ops.gelu(h)
    o = a @ w2 + b2
    loss = ops.mse(o, y)
    do = ops.mse_vjp(o, y)
    dw2, da = a.T @ do, do @ w2.T
    db2 = do.sum(axis=0)
    dh = ops.gelu_vjp(h, da)
    dw1 = x.T @ dh
    db1 = dh.sum(axis=0)
    return loss, [dw1, db1, dw2, db2]
