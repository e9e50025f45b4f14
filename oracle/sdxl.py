"""The SDXL UNet step and the SDXL (AutoencoderKL) VAE decoder, restated in numpy fp32 from the reference.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py). Parity unpinned: the reference's SDXL golden tensors are not
shipped (README.md:261-262) and its conv / norm / attention kernels live in the absent mako-common.

Follows src/image/sdxl.cpp: begin (:672-720: added conditioning from the pooled state and the image's sizes, each
transformer block's cross-attention K/V of the context), res_fwd (:722-740), trans_fwd (:742-796) and step
(:798-953: latents unpacked to a channels-last image scaled by 1/sqrt(sigma^2+1), the discrete timestep nearest to
sigma, time and label embeddings, one projection of silu(emb) for every residual block, input / middle / output
blocks with the skip concatenation, GroupNorm + SiLU + conv_out, eps repacked as tokens). The VAE decoder follows
src/image/engine.cpp:862-954 with res_block (:732-746) and vae_attention (:748-778) for the AutoencoderKL layout
(GroupNorm with bias, eps 1e-6).

Weights are named as the library's weight table names them (`unet_weight_shapes`, `vae_weight_shapes`); a 3x3
convolution is [Cout][3][3][Cin] (tap-major, channels-last), a 1x1 one [Cout][Cin].
"""

import math

import numpy as np

from . import ops as O

HEAD = 64
TOKENS_CTX = 77
ADDED = 2816


def unet_default_cfg(channels=(320, 640, 1280), depth=(0, 2, 10), layers=2, context_dim=2048, pooled_dim=1280):
    return {"channels": tuple(channels), "depth": tuple(depth), "layers": layers, "context_dim": context_dim,
            "pooled_dim": pooled_dim}


def unet_structure(cfg):
    """The block list: ('conv_in', cout) / ('res', name, cin, cout) / ('attn', name, c, depth) / ('down', name, c) /
    ('mid'), ('up', name, c), ('cat', skip_c), in the order the step runs them, with the skip pushes and pops of the
    reference's input / output blocks (sdxl.cpp:864-939)."""
    ch, dep, nl = cfg["channels"], cfg["depth"], cfg["layers"]
    ops = [("conv_in", "conv_in", ch[0]), ("push", ch[0])]
    skips = [ch[0]]
    c = ch[0]
    blk = 1
    for lvl in range(3):
        for k in range(nl):
            ops.append(("res", f"in{blk}.res", c, ch[lvl]))
            c = ch[lvl]
            if dep[lvl]:
                ops.append(("attn", f"in{blk}.attn", c, dep[lvl]))
            ops.append(("push", c))
            skips.append(c)
            blk += 1
        if lvl < 2:
            ops.append(("down", f"in{blk}.down", c))
            ops.append(("push", c))
            skips.append(c)
            blk += 1
    ops.append(("res", "mid.res0", c, c))
    ops.append(("attn", "mid.attn", c, dep[2]))
    ops.append(("res", "mid.res1", c, c))
    blk = 0
    for lvl in (2, 1, 0):
        for k in range(nl + 1):
            sc = skips.pop()
            ops.append(("cat", sc))
            ops.append(("res", f"out{blk}.res", c + sc, ch[lvl]))
            c = ch[lvl]
            if dep[lvl]:
                ops.append(("attn", f"out{blk}.attn", c, dep[lvl]))
            if lvl > 0 and k == nl:
                ops.append(("up", f"out{blk}.up", c))
            blk += 1
    return ops


def unet_weight_shapes(cfg):
    ch, ctx, pooled = cfg["channels"], cfg["context_dim"], cfg["pooled_dim"]
    temb = 4 * ch[0]
    s = {"time.lin1.w": (temb, ch[0]), "time.lin1.b": (temb,), "time.lin2.w": (temb, temb), "time.lin2.b": (temb,),
         "label.lin1.w": (temb, pooled + 6 * 256), "label.lin1.b": (temb,), "label.lin2.w": (temb, temb),
         "label.lin2.b": (temb,)}
    for op in unet_structure(cfg):
        if op[0] == "conv_in":
            s["conv_in.w"] = (op[2], 3, 3, 4)
            s["conv_in.b"] = (op[2],)
        elif op[0] == "res":
            _, n, cin, cout = op
            s.update({n + ".gn1.w": (cin,), n + ".gn1.b": (cin,), n + ".conv1.w": (cout, 3, 3, cin),
                      n + ".conv1.b": (cout,), n + ".emb.w": (cout, temb), n + ".emb.b": (cout,),
                      n + ".gn2.w": (cout,), n + ".gn2.b": (cout,), n + ".conv2.w": (cout, 3, 3, cout),
                      n + ".conv2.b": (cout,)})
            if cin != cout:
                s.update({n + ".skip.w": (cout, cin), n + ".skip.b": (cout,)})
        elif op[0] == "attn":
            _, n, c, d = op
            s.update({n + ".gn.w": (c,), n + ".gn.b": (c,), n + ".proj_in.w": (c, c), n + ".proj_in.b": (c,),
                      n + ".proj_out.w": (c, c), n + ".proj_out.b": (c,)})
            for j in range(d):
                p = f"{n}.b{j}."
                s.update({p + "ln1.w": (c,), p + "ln1.b": (c,), p + "qkv.w": (3 * c, c), p + "o1.w": (c, c),
                          p + "o1.b": (c,), p + "ln2.w": (c,), p + "ln2.b": (c,), p + "q2.w": (c, c),
                          p + "kv2.w": (2 * c, ctx), p + "o2.w": (c, c), p + "o2.b": (c,), p + "ln3.w": (c,),
                          p + "ln3.b": (c,), p + "ff1.w": (8 * c, c), p + "ff1.b": (8 * c,), p + "ff2.w": (c, 4 * c),
                          p + "ff2.b": (c,)})
        elif op[0] in ("down", "up"):
            _, n, c = op
            s.update({n + ".w": (c, 3, 3, c), n + ".b": (c,)})
    s.update({"out.gn.w": (ch[0],), "out.gn.b": (ch[0],), "out.conv.w": (4, 3, 3, ch[0]), "out.conv.b": (4,)})
    return s


def discrete_log_sigmas():
    """The SDXL schedule's 1000 levels (sdxl.cpp:130-139): betas linear in their square root 0.00085 -> 0.012."""
    cum = 1.0
    b0, b1 = math.sqrt(0.00085), math.sqrt(0.012)
    out = []
    for i in range(1000):
        b = b0 + (b1 - b0) * i / 999.0
        cum *= 1.0 - b * b
        out.append(np.float32(math.log(math.sqrt((1.0 - cum) / cum))))
    return np.array(out, np.float32)


def timestep(sigma):
    """Sdxl::timestep (sdxl.cpp:643-651): the level whose log-sigma is nearest (first on ties)."""
    ls = np.float32(math.log(sigma))
    table = discrete_log_sigmas()
    return int(np.argmin(np.abs(ls - table)))


def sinusoid(v, dim):
    """[cos(v f_i)..., sin(v f_i)...], f_i = 10000^(-i / (dim/2)) in float (sdxl.cpp:69-78)."""
    half = dim // 2
    i = np.arange(half, dtype=np.float32)
    f = np.exp(-np.log(np.float32(10000.0)) * i / np.float32(half)).astype(np.float32)
    a = (np.float32(v) * f).astype(np.float32)
    return np.concatenate([np.cos(a), np.sin(a)]).astype(np.float32)


def added_cond(pooled, gh, gw):
    """The added conditioning (sdxl.cpp:683-692): pooled state, then (H, W, 0, 0, H, W) as 256-wide sinusoids, the
    image size H = 16 gh, W = 16 gw."""
    H, W = float(16 * gh), float(16 * gw)
    return np.concatenate([np.asarray(pooled, np.float32)] + [sinusoid(v, 256) for v in (H, W, 0.0, 0.0, H, W)])


def unpack(tokens, gh, gw, scale, z=4, mean=None):
    """Tokens [gh*gw][4 z] (channel, row, column of a 2x2 patch) to the channels-last image [2gh][2gw][z]
    (sdxl.cpp:80-87), each value times `scale` (a number, or one per token value) plus `mean` (one per token value,
    Engine::decode's latent statistics, engine.cpp:890-898)."""
    t = np.asarray(tokens, np.float32).reshape(gh * gw, 4 * z)
    t = t * np.asarray(scale, np.float32)
    if mean is not None:
        t = t + np.asarray(mean, np.float32)
    t = t.astype(np.float32).reshape(gh, gw, z, 2, 2)
    return t.transpose(0, 3, 1, 4, 2).reshape(2 * gh, 2 * gw, z).astype(np.float32)


def pack(img, gh, gw):
    """The inverse of unpack (sdxl.cpp:946-952)."""
    return np.asarray(img, np.float32).reshape(gh, 2, gw, 2, 4).transpose(0, 2, 4, 1, 3).reshape(gh * gw, 16)


def _conv(W, n, x, stride=1):
    w = W[n + ".w"]
    if w.ndim == 2:
        return O.conv2d_nhwc(x[None], w[:, None, :], 1, 1, W.get(n + ".b"))[0]
    cout = w.shape[0]
    return O.conv2d_nhwc(x[None], w.reshape(cout, 9, w.shape[3]), stride, 9, W.get(n + ".b"))[0]


def _layer_norm(x, g, b, eps=1e-5):
    x64 = x.astype(np.float64)
    m = x64.mean(-1, keepdims=True)
    v = ((x64 - m) ** 2).mean(-1, keepdims=True)
    return (((x64 - m) / np.sqrt(v + eps)) * g + b).astype(np.float32)


def res_fwd(W, n, x, eo_row, eps=1e-5):
    """Sdxl::res_fwd (sdxl.cpp:722-740) on one image x [H][W][cin] (fp32); eo_row: this block's emb projection."""
    t = O.group_norm_nhwc(x[None], W[n + ".gn1.w"], W[n + ".gn1.b"], 32, eps, True)[0]
    t = _conv(W, n + ".conv1", t) + eo_row
    t = O.group_norm_nhwc(t[None], W[n + ".gn2.w"], W[n + ".gn2.b"], 32, eps, True)[0]
    y = _conv(W, n + ".conv2", t)
    return (y + (_conv(W, n + ".skip", x) if n + ".skip.w" in W else x)).astype(np.float32)


def trans_fwd(W, n, x, depth, kv):
    """Sdxl::trans_fwd (sdxl.cpp:742-796) on x [H][W][c]; kv: per block (k, v) [heads][S][64] of the context."""
    Hh, Ww, c = x.shape
    heads = c // HEAD
    xt = x.reshape(-1, c)
    xn = O.group_norm_nhwc(x[None], W[n + ".gn.w"], W[n + ".gn.b"], 32, 1e-6, False)[0].reshape(-1, c)
    hs = O.linear(xn, W[n + ".proj_in.w"], W[n + ".proj_in.b"])
    for j in range(depth):
        p = f"{n}.b{j}."
        hn = _layer_norm(hs, W[p + "ln1.w"], W[p + "ln1.b"])
        qkv = O.linear(hn, W[p + "qkv.w"])
        q, k, v = (qkv[:, i * c:(i + 1) * c].reshape(-1, heads, HEAD).transpose(1, 0, 2) for i in range(3))
        att = O.attention(q, k, v).transpose(1, 0, 2).reshape(-1, c)
        hs = hs + O.linear(att, W[p + "o1.w"], W[p + "o1.b"])
        hn = _layer_norm(hs, W[p + "ln2.w"], W[p + "ln2.b"])
        q = O.linear(hn, W[p + "q2.w"]).reshape(-1, heads, HEAD).transpose(1, 0, 2)
        att = O.attention(q, kv[j][0], kv[j][1]).transpose(1, 0, 2).reshape(-1, c)
        hs = hs + O.linear(att, W[p + "o2.w"], W[p + "o2.b"])
        hn = _layer_norm(hs, W[p + "ln3.w"], W[p + "ln3.b"])
        ff = O.linear(hn, W[p + "ff1.w"], W[p + "ff1.b"])
        m = ff[:, :4 * c] * O.gelu_erf(ff[:, 4 * c:])
        hs = hs + O.linear(m, W[p + "ff2.w"], W[p + "ff2.b"])
    out = O.linear(hs, W[n + ".proj_out.w"], W[n + ".proj_out.b"]) + xt
    return out.reshape(Hh, Ww, c).astype(np.float32)


def unet_begin(cfg, W, context, pooled, gh, gw):
    """Sdxl::begin (sdxl.cpp:672-720): the added conditioning and every transformer block's context K/V."""
    y = added_cond(pooled, gh, gw)
    kv = {}
    for op in unet_structure(cfg):
        if op[0] == "attn":
            _, n, c, d = op
            heads = c // HEAD
            blocks = []
            for j in range(d):
                kvm = O.linear(context, W[f"{n}.b{j}.kv2.w"])
                k = kvm[:, :c].reshape(-1, heads, HEAD).transpose(1, 0, 2)
                v = kvm[:, c:].reshape(-1, heads, HEAD).transpose(1, 0, 2)
                blocks.append((k, v))
            kv[n] = blocks
    return {"y": y, "kv": kv, "gh": gh, "gw": gw}


def unet_step(cfg, W, state, tokens, sigma, probe=None):
    """Sdxl::step (sdxl.cpp:798-953): predicted noise as tokens [gh*gw][16]."""
    pr = probe or (lambda name, a: None)
    gh, gw = state["gh"], state["gw"]
    x = unpack(tokens, gh, gw, 1.0 / math.sqrt(sigma * sigma + 1.0))
    te = sinusoid(float(timestep(sigma)), cfg["channels"][0])[None]
    e1 = O.silu(O.linear(te, W["time.lin1.w"], W["time.lin1.b"]))
    emb = O.linear(e1, W["time.lin2.w"], W["time.lin2.b"])
    pr("temb", emb)
    l1 = O.silu(O.linear(state["y"][None], W["label.lin1.w"], W["label.lin1.b"]))
    l2 = O.linear(l1, W["label.lin2.w"], W["label.lin2.b"])
    se = O.silu(emb + l2)[0]
    skips = []
    h = x
    for op in unet_structure(cfg):
        kind = op[0]
        if kind == "conv_in":
            h = _conv(W, "conv_in", h)
        elif kind == "push":
            skips.append(h)
        elif kind == "res":
            n = op[1]
            eo = O.linear(se[None], W[n + ".emb.w"], W[n + ".emb.b"])[0]
            h = res_fwd(W, n, h, eo)
        elif kind == "attn":
            h = trans_fwd(W, op[1], h, op[3], state["kv"][op[1]])
        elif kind == "down":
            h = _conv(W, op[1], h, stride=2)
        elif kind == "cat":
            h = np.concatenate([h, skips.pop()], axis=-1)
        elif kind == "up":
            h = _conv(W, op[1], O.upsample2x_nhwc(h[None])[0])
        if kind in ("res", "attn", "down", "up", "conv_in"):
            pr(op[1], h)
    t = O.group_norm_nhwc(h[None], W["out.gn.w"], W["out.gn.b"], 32, 1e-5, True)[0]
    eps = _conv(W, "out.conv", t)
    return pack(eps, gh, gw)


# ---------------------------------------------------------------------------------------------- VAE decoder


def vae_default_cfg(channels=(128, 256, 512, 512), layers=2, latent=4, scale=0.13025):
    return {"channels": tuple(channels), "layers": layers, "latent": latent, "scale": scale}


def vae_structure(cfg):
    """AutoencoderKL decoder: conv_in to the widest width, mid (res, attention, res), then up levels from the widest
    down, layers + 1 residual blocks each, a 2x upsample + conv after every level but the last (engine.cpp:900-941)."""
    ch = cfg["channels"]
    c = ch[-1]
    ops = [("post_quant",), ("conv_in", c), ("res", "mid.res0", c, c), ("attn", "mid.attn", c), ("res", "mid.res1", c, c)]
    n_lvl = len(ch)
    for i, lvl in enumerate(reversed(range(n_lvl))):
        for k in range(cfg["layers"] + 1):
            ops.append(("res", f"up{i}.res{k}", c, ch[lvl]))
            c = ch[lvl]
        if i < n_lvl - 1:
            ops.append(("up", f"up{i}.up", c))
    return ops


def vae_weight_shapes(cfg):
    z = cfg["latent"]
    s = {"post_quant.w": (z, z), "post_quant.b": (z,)}
    for op in vae_structure(cfg):
        if op[0] == "conv_in":
            s.update({"conv_in.w": (op[1], 3, 3, z), "conv_in.b": (op[1],)})
        elif op[0] == "res":
            _, n, cin, cout = op
            s.update({n + ".gn1.w": (cin,), n + ".gn1.b": (cin,), n + ".conv1.w": (cout, 3, 3, cin),
                      n + ".conv1.b": (cout,), n + ".gn2.w": (cout,), n + ".gn2.b": (cout,),
                      n + ".conv2.w": (cout, 3, 3, cout), n + ".conv2.b": (cout,)})
            if cin != cout:
                s.update({n + ".skip.w": (cout, cin), n + ".skip.b": (cout,)})
        elif op[0] == "attn":
            c = op[2]
            s.update({"mid.attn.gn.w": (c,), "mid.attn.gn.b": (c,), "mid.attn.qkv.w": (3 * c, c),
                      "mid.attn.qkv.b": (3 * c,), "mid.attn.proj.w": (c, c), "mid.attn.proj.b": (c,)})
        elif op[0] == "up":
            c = op[2]
            s.update({op[1] + ".w": (c, 3, 3, c), op[1] + ".b": (c,)})
    c0 = cfg["channels"][0]
    s.update({"out.gn.w": (c0,), "out.gn.b": (c0,), "out.conv.w": (3, 3, 3, c0), "out.conv.b": (3,)})
    return s


def vae_decode(cfg, W, tokens, gh, gw, probe=None, stats=None):
    """Engine::decode (engine.cpp:862-954), AutoencoderKL layout: tokens [gh*gw][4 latent] to RGBA [16gh][16gw][4] in
    [-1, 1]. The latents are tokens / scale, or with stats = (mean, std) per token value tokens * std + mean."""
    pr = probe or (lambda name, a: None)
    z = cfg["latent"]
    if stats is None:
        x = unpack(tokens, gh, gw, 1.0 / cfg["scale"], z)
    else:
        x = unpack(tokens, gh, gw, stats[1], z, stats[0])
    h = _conv(W, "post_quant", x)
    for op in vae_structure(cfg)[1:]:
        kind = op[0]
        if kind == "conv_in":
            h = _conv(W, "conv_in", h)
        elif kind == "res":
            h = res_fwd(W, op[1], h, 0.0, eps=1e-6)
        elif kind == "attn":
            Hh, Ww, c = h.shape
            t = O.group_norm_nhwc(h[None], W["mid.attn.gn.w"], W["mid.attn.gn.b"], 32, 1e-6, False)[0].reshape(-1, c)
            qkv = O.linear(t, W["mid.attn.qkv.w"], W["mid.attn.qkv.b"])
            q, k, v = (qkv[:, i * c:(i + 1) * c][None] for i in range(3))
            att = O.attention(q, k, v)[0]
            h = h + O.linear(att, W["mid.attn.proj.w"], W["mid.attn.proj.b"]).reshape(Hh, Ww, c)
        elif kind == "up":
            h = _conv(W, op[1], O.upsample2x_nhwc(h[None])[0])
        pr(op[1] if len(op) > 1 and isinstance(op[1], str) else kind, h)
    t = O.group_norm_nhwc(h[None], W["out.gn.w"], W["out.gn.b"], 32, 1e-6, True)[0]
    rgb = np.clip(_conv(W, "out.conv", t), -1.0, 1.0)
    return np.concatenate([rgb, np.ones(rgb.shape[:2] + (1,), np.float32)], axis=-1)
