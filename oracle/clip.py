"""The SDXL text encoders (CLIP ViT-L and OpenCLIP bigG) and the prompt embeddings built from them, restated in numpy.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py). Parity unpinned: the reference ships no text-encoder golden tensors
and its LayerNorm / GEMM / attention kernels live in the absent mako-common.

Follows src/image/sdxl.cpp:459-546 (Sdxl::encode_clip): a chunk of 77 token ids; token embeddings (F16 in the
checkpoint, read exactly) plus the positional embeddings; per layer a pre-LayerNorm block: LN1, the fused q | k | v
projection with bias, attention in heads of 64 with the runtime's mask argument UINT32_MAX (:501), which
docs/architecture.md:92 calls causal (a token sees itself and the tokens before it), the output projection with
bias, residual; LN2, fc1 with bias, quick GELU x sigmoid(1.702 x) (ViT-L) or the erf GELU (bigG) (:508), fc2 with
bias, residual. The hidden state is the output of the second to last layer (:512-515). bigG's pooled state is its
final state at the first end token (49407), LayerNormed with ln_final (eps 1e-5) and multiplied by the projection as
stored, [E][1280] (:521-541). LayerNorm eps is 1e-5 throughout (CLIP's). Sdxl::prompt_embeddings (:599-639): per
chunk ViT-L's and bigG's hidden states side by side (768 + 1280 = 2048 per token), a weighted token's states moved
away from the empty prompt's by its weight, (z - e) w + e, and the pooled state of the first chunk.

The reference feeds every projection its input split into a bf16 part and the bf16 rounding of what that part left
out (docs/architecture.md:9-11): for weights in bf16 that is the product of the fp32 input to within ~2^-16. The
oracle multiplies fp32 inputs by the bf16 weights in float64.

Weights are named as the library's weight table names them (`weight_shapes`).
"""

import numpy as np

TOKENS = 77
HEAD = 64
POOLED = 1280
START, END = 49406, 49407
EPS = 1e-5


def default_cfg(which, vocab=49408, **over):
    """which 0: ViT-L (12 layers, 768, quick GELU); 1: OpenCLIP bigG (32 layers, 1280, erf GELU, pooled)."""
    if which == 0:
        c = {"which": 0, "width": 768, "heads": 12, "layers": 12, "ffn": 3072, "vocab": vocab}
    else:
        c = {"which": 1, "width": 1280, "heads": 20, "layers": 32, "ffn": 5120, "vocab": vocab}
    c.update(over)
    return c


def weight_shapes(cfg):
    E, F = cfg["width"], cfg["ffn"]
    s = {"tok": (cfg["vocab"], E), "pos": (TOKENS, E)}
    for i in range(cfg["layers"]):
        p = f"l{i}."
        s.update({p + "ln1.w": (E,), p + "ln1.b": (E,), p + "qkv.w": (3 * E, E), p + "qkv.b": (3 * E,),
                  p + "o.w": (E, E), p + "o.b": (E,), p + "ln2.w": (E,), p + "ln2.b": (E,),
                  p + "fc1.w": (F, E), p + "fc1.b": (F,), p + "fc2.w": (E, F), p + "fc2.b": (E,)})
    if cfg["which"] == 1:
        s.update({"lnf.w": (E,), "lnf.b": (E,), "proj": (E, POOLED)})
    return s


def layer_norm(x, g, b, eps=EPS):
    x = x.astype(np.float64)
    m = x.mean(-1, keepdims=True)
    v = ((x - m) ** 2).mean(-1, keepdims=True)
    return (x - m) / np.sqrt(v + eps) * g + b


def _lin(x, w, b):
    return x.astype(np.float64) @ w.astype(np.float64).T + b


def _gelu_erf(x):
    from math import erf

    return 0.5 * x * (1.0 + np.vectorize(erf)(x / np.sqrt(2.0)))


def encode(cfg, W, ids, probe=None):
    """One chunk: ids [77] -> (hidden [77][E] float32, pooled [1280] float32 for bigG else None)."""
    ids = np.asarray(ids)
    assert ids.shape == (TOKENS,)
    E, H = cfg["width"], cfg["heads"]
    x = W["tok"][ids].astype(np.float64) + W["pos"]
    causal = np.tril(np.ones((TOKENS, TOKENS), bool))
    pooled_wanted = cfg["which"] == 1
    n_run = cfg["layers"] if pooled_wanted else cfg["layers"] - 1
    hidden = None
    for i in range(n_run):
        p = f"l{i}."
        xn = layer_norm(x, W[p + "ln1.w"], W[p + "ln1.b"])
        qkv = _lin(xn, W[p + "qkv.w"], W[p + "qkv.b"])
        q, k, v = (qkv[:, j * E:(j + 1) * E].reshape(TOKENS, H, HEAD).transpose(1, 0, 2) for j in range(3))
        s = q @ k.transpose(0, 2, 1) / np.sqrt(HEAD)
        s = np.where(causal, s, -np.inf)
        s = np.exp(s - s.max(-1, keepdims=True))
        att = (s / s.sum(-1, keepdims=True)) @ v
        x = x + _lin(att.transpose(1, 0, 2).reshape(TOKENS, E), W[p + "o.w"], W[p + "o.b"])
        xn = layer_norm(x, W[p + "ln2.w"], W[p + "ln2.b"])
        h = _lin(xn, W[p + "fc1.w"], W[p + "fc1.b"])
        h = h / (1.0 + np.exp(-1.702 * h)) if cfg["which"] == 0 else _gelu_erf(h)
        x = x + _lin(h, W[p + "fc2.w"], W[p + "fc2.b"])
        if probe:
            probe(f"layer{i}", x.astype(np.float32))
        if i + 2 == cfg["layers"]:
            hidden = x.astype(np.float32)
    pooled = None
    if pooled_wanted:
        eos = int(np.argmax(ids == END))
        assert ids[eos] == END, "a chunk without its end token"
        r = layer_norm(x[eos], W["lnf.w"], W["lnf.b"])
        pooled = (r @ W["proj"].astype(np.float64)).astype(np.float32)
    return hidden, pooled


def empty_ids(pad):
    """The empty prompt's chunk: start, end, then padding (sdxl.cpp:45-51; ViT-L pads with the end token, bigG 0)."""
    ids = np.full(TOKENS, pad, np.int32)
    ids[0], ids[1] = START, END
    return ids


def prompt_embeddings(cfg_l, W_l, cfg_g, W_g, ids_l, ids_g, weights):
    """Chunks of ids [n][77] for each encoder and per-token weights [n][77] -> (context [n * 77][2048], pooled)."""
    ids_l, ids_g, weights = np.asarray(ids_l), np.asarray(ids_g), np.asarray(weights, np.float32)
    weighted = bool((weights != 1.0).any())
    e_l = encode(cfg_l, W_l, empty_ids(END))[0] if weighted else None
    e_g = encode(cfg_g, W_g, empty_ids(0))[0] if weighted else None
    out, pooled = [], None
    for k in range(ids_l.shape[0]):
        zl = encode(cfg_l, W_l, ids_l[k])[0]
        zg, pg = encode(cfg_g, W_g, ids_g[k])
        if k == 0:
            pooled = pg
        if weighted:
            w = weights[k][:, None]
            zl = np.where(w != 1.0, (zl - e_l) * w + e_l, zl)
            zg = np.where(w != 1.0, (zg - e_g) * w + e_g, zg)
        out.append(np.concatenate([zl, zg], 1))
    return np.concatenate(out, 0).astype(np.float32), pooled
