"""The Qwen-Image-style MMDiT denoiser step, restated in numpy from the reference.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py). Parity unpinned: no golden tensors of this path ship with the
reference (README.md:261-262).

Two variants, selected by `cfg["variant"]`:

* "ref21": the reference's own math (src/image/qwen_image.cpp:144-293): one weight set for text and image rows; one
  shared modulation Linear D -> 4D applied to silu(temb) of two timesteps (row 0: sigma, the image; row 1: t = 0, the
  text; :196-205, :222); LayerNorm x (1 + scale) without shift (src/kernels/image.metal:33-53); tanh-squashed gates
  (:56-65); SwiGLU FFN (:277-280); condition-causal attention (the runtime's `block = S`, :271: a text row at
  position p attends to keys 0..p, causal among the text and never to an image key, so the text K/V is cached after
  the first step, :251-262; the same argument is UINT32_MAX for the CLIP encoders, sdxl.cpp:501, which
  docs/architecture.md:92 calls causal, and 0 for unmasked attention, sdxl.cpp:773); RoPE positions text (t, t, t), image (S, y - ceil(h/2), x - ceil(w/2))
  (:134-141); no biases.
* "qwen1": the Qwen-Image(-1) shape BASELINE.json names: separate text and image weights with biases; per-block
  AdaLN Linear D -> 6D per stream ([shift1, scale1, gate1, shift2, scale2, gate2]); x (1 + scale) + shift; plain
  gates; GELU-tanh FFN; fully joint attention; text RoPE positions m + t on all three axes with
  m = max(h // 2, w // 2), image (0, y - ceil(h/2), x - ceil(w/2)); txt_in = RMSNorm -> Linear; norm_out with
  [scale, shift].

Shapes: latents [N][64] (N = h * w 2x2-patch tokens), prompt [S][text_dim], weights as named by `weight_shapes`.
Weights are given as fp32 arrays (bf16-rounded where the device stores bf16). Activations stay fp32 throughout.
"""

import numpy as np

from . import ops as O

HEAD_DIM = 128
LATENT = 64
TIME_DIM = 256
EPS = 1e-6


def default_cfg(variant="qwen1", D=3072, heads=24, F=12288, blocks=60, text_dim=3584):
    return {"variant": variant, "D": D, "heads": heads, "F": F, "blocks": blocks, "text_dim": text_dim}


def weight_shapes(cfg):
    """Name -> shape of every weight, in the order the library stores them."""
    D, F, T, nb = cfg["D"], cfg["F"], cfg["text_dim"], cfg["blocks"]
    s = {}
    if cfg["variant"] == "qwen1":
        s.update({"time.lin1.w": (D, TIME_DIM), "time.lin1.b": (D,), "time.lin2.w": (D, D), "time.lin2.b": (D,),
                  "img_in.w": (D, LATENT), "img_in.b": (D,), "txt_norm.w": (T,), "txt_in.w": (D, T),
                  "txt_in.b": (D,), "norm_out.w": (2 * D, D), "norm_out.b": (2 * D,), "proj_out.w": (LATENT, D),
                  "proj_out.b": (LATENT,)})
        for i in range(nb):
            for st in ("img", "txt"):
                p = f"blk{i}.{st}."
                s.update({p + "mod.w": (6 * D, D), p + "mod.b": (6 * D,), p + "qkv.w": (3 * D, D),
                          p + "qkv.b": (3 * D,), p + "norm_q": (HEAD_DIM,), p + "norm_k": (HEAD_DIM,),
                          p + "o.w": (D, D), p + "o.b": (D,), p + "ff1.w": (F, D), p + "ff1.b": (F,),
                          p + "ff2.w": (D, F), p + "ff2.b": (D,)})
    else:
        s.update({"time.lin1.w": (D, TIME_DIM), "time.lin2.w": (D, D), "mod.w": (4 * D, D), "img_in.w": (D, LATENT),
                  "txt_norm.w": (T,), "txt_in1.w": (D, T), "txt_in2.w": (D, D), "norm_out.w": (D, D),
                  "proj_out.w": (LATENT, D)})
        for i in range(nb):
            p = f"blk{i}."
            s.update({p + "qkv.w": (3 * D, D), p + "norm_q": (HEAD_DIM,), p + "norm_k": (HEAD_DIM,),
                      p + "o.w": (D, D), p + "gate_up.w": (2 * F, D), p + "down.w": (D, F)})
    return s


def _rope_axes(pos):
    """rope3 (qwen_image.cpp:31-45): 8 pairs on the frame axis, then 28 each on height and width, theta 10000.
    pos [L][3] integer positions -> table [L][64][2] of (cos, sin)."""
    dims = (16, 56, 56)
    angs = []
    for a, d in enumerate(dims):
        j = np.arange(d // 2, dtype=np.float32)
        inv = (1.0 / np.power(np.float32(10000.0), 2.0 * j / np.float32(d))).astype(np.float32)
        angs.append(pos[:, a:a + 1].astype(np.float32) * inv[None, :])
    ang = np.concatenate(angs, axis=1).astype(np.float32)
    return np.stack([np.cos(ang), np.sin(ang)], axis=-1).astype(np.float32)


def rope_table(cfg, S, h, w):
    """The RoPE table of the joint sequence [text S rows, image h*w rows] (qwen_image.cpp:134-141 for ref21)."""
    y, x = np.meshgrid(np.arange(h), np.arange(w), indexing="ij")
    y = y.reshape(-1) - (h - h // 2)
    x = x.reshape(-1) - (w - w // 2)
    t = np.arange(S)
    if cfg["variant"] == "ref21":
        txt = np.stack([t, t, t], 1)
        img = np.stack([np.full_like(y, S), y, x], 1)
    else:
        m = max(h // 2, w // 2)
        txt = np.stack([t + m] * 3, 1)
        img = np.stack([np.zeros_like(y), y, x], 1)
    return _rope_axes(np.concatenate([txt, img], 0))


def time_embedding(W, sigma):
    """temb = lin2(silu(lin1(sinusoid(sigma)))) (qwen_image.cpp:179-202; time_text_embed)."""
    tp = O.timestep_sinusoid(sigma, TIME_DIM)[None]
    h = O.silu(O.linear(tp, W["time.lin1.w"], W.get("time.lin1.b")))
    return O.linear(h, W["time.lin2.w"], W.get("time.lin2.b"))[0]


def _heads(x, H):
    """[rows][H*128] -> [H][rows][128]."""
    return x.reshape(x.shape[0], H, HEAD_DIM).transpose(1, 0, 2)


def _unheads(x):
    return x.transpose(1, 0, 2).reshape(x.shape[1], -1)


def text_in(cfg, W, prompt):
    """The text stream's input rows (qwen_image.cpp:206-214 for ref21)."""
    xn = O.rms_norm(prompt, W["txt_norm.w"], EPS)
    if cfg["variant"] == "qwen1":
        return O.linear(xn, W["txt_in.w"], W["txt_in.b"])
    return O.linear(O.gelu_tanh(O.linear(xn, W["txt_in1.w"])), W["txt_in2.w"])


def block_qwen1(cfg, W, i, x_txt, x_img, st, rope):
    """One Qwen-Image-1 double-stream block on one sample; st = silu(temb). Returns the new (x_txt, x_img)."""
    H, D = cfg["heads"], cfg["D"]
    S = x_txt.shape[0]
    qs, ks, vs, mods = [], [], [], {}
    for name, x, r in (("txt", x_txt, rope[:S]), ("img", x_img, rope[S:])):
        p = f"blk{i}.{name}."
        mod = O.linear(st[None], W[p + "mod.w"], W[p + "mod.b"])[0].reshape(6, D)
        mods[name] = mod
        xn = O.ln_modulate(x, mod[1], mod[0], EPS)
        qkv = O.linear(xn, W[p + "qkv.w"], W[p + "qkv.b"])
        q, k, v = (_heads(qkv[:, j * D:(j + 1) * D], H) for j in range(3))
        qs.append(O.rope_pairs(O.rms_norm(q, W[p + "norm_q"], EPS), r))
        ks.append(O.rope_pairs(O.rms_norm(k, W[p + "norm_k"], EPS), r))
        vs.append(v)
    att = _unheads(O.attention(np.concatenate(qs, 1), np.concatenate(ks, 1), np.concatenate(vs, 1)))
    out = []
    for name, x, a in (("txt", x_txt, att[:S]), ("img", x_img, att[S:])):
        p = f"blk{i}.{name}."
        mod = mods[name]
        x = x + mod[2] * O.linear(a, W[p + "o.w"], W[p + "o.b"])
        xn = O.ln_modulate(x, mod[4], mod[3], EPS)
        hdn = O.gelu_tanh(O.linear(xn, W[p + "ff1.w"], W[p + "ff1.b"]))
        x = x + mod[5] * O.linear(hdn, W[p + "ff2.w"], W[p + "ff2.b"])
        out.append(x.astype(np.float32))
    return out[0], out[1]


def block_ref21(cfg, W, i, x, split, mod, rope, kv_cache=None):
    """One reference block (qwen_image.cpp:219-284) on the rows x ([text rows if any][image rows]).

    split: text rows at the top of x (S on the first step, 0 later). mod [2][4D]: row 0 the image's
    [scale1, gate1, scale2, gate2], row 1 the text's. kv_cache: dict of this block's text K/V (filled on the first
    step, read on later ones), or None to run without caching (all rows present)."""
    H, D, F = cfg["heads"], cfg["D"], cfg["F"]
    T = x.shape[0]
    rowmod = np.where(np.arange(T)[:, None] < split, mod[1][None, :], mod[0][None, :])
    xn = O.ln_modulate(x, rowmod[:, 0:D], None, EPS)
    qkv = O.linear(xn, W[f"blk{i}.qkv.w"])
    q, k, v = (_heads(qkv[:, j * D:(j + 1) * D], H) for j in range(3))
    q = O.rope_pairs(O.rms_norm(q, W[f"blk{i}.norm_q"], EPS), rope)
    k = O.rope_pairs(O.rms_norm(k, W[f"blk{i}.norm_k"], EPS), rope)
    if kv_cache is not None and split == 0:  # later steps: text K/V from the first
        k = np.concatenate([kv_cache["k"], k], 1)
        v = np.concatenate([kv_cache["v"], v], 1)
        S = kv_cache["k"].shape[1]
    else:
        S = split
        if kv_cache is not None:
            kv_cache["k"], kv_cache["v"] = k[:, :S].copy(), v[:, :S].copy()
    Lk = k.shape[1]
    qpos = np.arange(Lk - T, Lk)
    # Condition-causal: a text query at position p sees keys 0..p (never an image key); image queries see all.
    mask = (qpos[:, None] >= S) | (np.arange(Lk)[None, :] <= qpos[:, None])
    att = _unheads(O.attention(q, k, v, mask))
    x = x + np.tanh(rowmod[:, D:2 * D]) * O.linear(att, W[f"blk{i}.o.w"])
    xn = O.ln_modulate(x, rowmod[:, 2 * D:3 * D], None, EPS)
    gu = O.linear(xn, W[f"blk{i}.gate_up.w"])
    m = O.silu(gu[:, :F]) * gu[:, F:]
    x = x + np.tanh(rowmod[:, 3 * D:4 * D]) * O.linear(m, W[f"blk{i}.down.w"])
    return x.astype(np.float32)


def step(cfg, W, latents, prompt, sigma, h, w, state=None, probe=None, blocks=None):
    """One denoiser step for one sample: the velocity [N][64] (Engine::step, engine.hpp:165-166).

    state: for ref21, a dict carried between steps of one generation (text rows and K/V cache); None runs the full
    sequence every step. probe(name, array): called with named stages like the reference's probes
    (qwen_image.cpp:200-287). blocks: how many blocks to run (default all)."""
    D = cfg["D"]
    nb = cfg["blocks"] if blocks is None else blocks
    N = h * w
    S = prompt.shape[0]
    rope = rope_table(cfg, S, h, w)
    pr = probe or (lambda name, a: None)
    if cfg["variant"] == "qwen1":
        temb = time_embedding(W, sigma)
        pr("temb", temb)
        st = O.silu(temb)
        x_txt = text_in(cfg, W, prompt)
        pr("txt_in", x_txt)
        x_img = O.linear(latents, W["img_in.w"], W["img_in.b"])
        pr("img_in", x_img)
        for i in range(nb):
            x_txt, x_img = block_qwen1(cfg, W, i, x_txt, x_img, st, rope)
            pr(f"block{i}", np.concatenate([x_txt, x_img], 0))
        so = O.linear(st[None], W["norm_out.w"], W["norm_out.b"])[0]
        xn = O.ln_modulate(x_img, so[:D], so[D:], EPS)
        pr("norm_out", xn)
        return O.linear(xn, W["proj_out.w"], W["proj_out.b"])
    # ref21
    temb = np.stack([time_embedding(W, sigma), time_embedding(W, 0.0)])
    pr("temb", temb)
    st = O.silu(temb)
    mod = O.linear(st, W["mod.w"])
    pr("modulation", mod)
    omod = O.linear(st, W["norm_out.w"])
    first = state is None or "steps" not in state or state["steps"] == 0
    if state is not None:
        state["steps"] = state.get("steps", 0) + 1
        state.setdefault("kv", [dict() for _ in range(cfg["blocks"])])
    x_img = O.linear(latents, W["img_in.w"])
    pr("img_in", x_img)
    if first:
        x_txt = text_in(cfg, W, prompt)
        pr("txt_in", x_txt)
        x = np.concatenate([x_txt, x_img], 0)
        split, r = S, rope
    else:
        x, split, r = x_img, 0, rope[S:]
    for i in range(nb):
        x = block_ref21(cfg, W, i, x, split, mod, r, state["kv"][i] if state is not None else None)
        pr(f"block{i}", x)
    rows = np.arange(x.shape[0])[:, None] < split
    xn = O.ln_modulate(x, np.where(rows, omod[1][None], omod[0][None]), None, EPS)
    pr("norm_out", xn)
    return O.linear(xn, W["proj_out.w"])[x.shape[0] - N:]
