"""SDXL's text encoders (mkb_clip_*, mkb_sdxl_prompt_embeddings) against the numpy oracle (oracle/clip.py).

* ViT-L at its full size (768 wide, 12 heads, 12 layers, FFN 3072, quick GELU) and bigG at its full width (1280, 20
  heads, FFN 5120, erf GELU) over fewer layers: every layer's output (cosine >= 0.9999), the hidden states (the
  second to last layer's, rel-RMS < 5e-3) and bigG's pooled state.
* Causality: changing a later token leaves every earlier token's states bit for bit unchanged.
* The prompt embeddings of weighted chunks (two chunks, weights 0.7 and 1.3 on some tokens), side by side.
* The checkpoint names of both encoders (Sdxl::load_clip, sdxl.cpp:154-237) and rejected inputs.

Random weights N(0, 0.02) with the token and position tables at N(0, 0.5) scale, so the residual stream is O(1).
The reference's own bar on the encoders' states, the weighted conditioning and the pooled state is rel-RMS < 0.01
(tests/sdxl_ref_test.cpp:203-218); these hold half of it."""

import os
import sys

import numpy as np
import pytest

from oracle import clip as OC
from oracle import rng

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from st_files import write_safetensors  # noqa: E402

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.astype(np.float64), b.astype(np.float64)
    return float(np.sqrt(((a - b) ** 2).sum() / (b ** 2).sum()))


def _cos(a, b):
    a, b = a.astype(np.float64).ravel(), b.astype(np.float64).ravel()
    return float(a @ b / np.sqrt((a @ a) * (b @ b)))


def _model(mkimage, cfg, seed):
    c = mkimage.Clip(cfg)
    c.init_random(seed, 0.02)
    for name in ("tok", "pos"):  # embeddings of unit scale, as trained ones roughly are
        shape = dict(c.weight_names())[name]
        c.write_weight(name, rng.normal(rng.tensor_key(seed, 7 if name == "tok" else 8), int(np.prod(shape)))
                       .reshape(shape) * 0.5)
    return c


def _ocfg(cfg):
    return OC.default_cfg(cfg.which, vocab=cfg.vocab, width=cfg.width, heads=cfg.heads, layers=cfg.layers,
                          ffn=cfg.ffn)


def _ids(seed, n_words, pad):
    """A chunk as Sdxl::chunks makes one: start, words, end, padding."""
    words = np.random.RandomState(seed).randint(1, 49000, n_words).astype(np.int32)
    ids = np.full(77, pad, np.int32)
    ids[0] = OC.START
    ids[1:1 + n_words] = words
    ids[1 + n_words] = OC.END
    return ids


@pytest.mark.parametrize("which,layers", [(0, 12), (1, 4)])
def test_clip_encoder_matches_oracle(cuda, which, layers):
    import mkimage

    cfg = mkimage.ClipConfig.sdxl(which, layers=layers, max_chunks=2)
    c = _model(mkimage, cfg, 31 + which)
    W = c.weights()
    ids = _ids(5 + which, 11, OC.END if which == 0 else 0)
    got = {}
    c.set_probe(lambda name, layer, a: got.__setitem__(layer, a))
    hidden, pooled = c.encode(ids[None])
    c.set_probe(None)
    c.close()
    want = {}
    ref_h, ref_p = OC.encode(_ocfg(cfg), W, ids, probe=lambda n, a: want.__setitem__(int(n[5:]), a))
    for layer, a in want.items():
        assert _cos(got[layer], a) >= 0.9999, (layer, _cos(got[layer], a))
    assert _rel(hidden, ref_h) < 5e-3, _rel(hidden, ref_h)
    if which == 1:
        assert _rel(pooled[0], ref_p) < 5e-3, _rel(pooled[0], ref_p)
    else:
        assert pooled is None


def test_clip_is_causal(cuda):
    import mkimage

    cfg = mkimage.ClipConfig.sdxl(1, layers=3, max_chunks=2)
    c = _model(mkimage, cfg, 41)
    a = _ids(9, 20, 0)
    b = a.copy()
    b[30] = 777  # a token after the end: only rows >= 30 may change
    ha, _ = c.encode(np.stack([a, b]))
    c.close()
    assert np.array_equal(ha[:30], ha[77:77 + 30])
    assert not np.array_equal(ha[30:77], ha[77 + 30:])


def test_prompt_embeddings_weighted_chunks(cuda):
    import mkimage

    cl = mkimage.ClipConfig(which=0, width=256, heads=4, layers=3, ffn=512, max_chunks=2)
    cg = mkimage.ClipConfig(which=1, width=384, heads=6, layers=3, ffn=768, max_chunks=2)
    L, G = _model(mkimage, cl, 51), _model(mkimage, cg, 52)
    ids_l = np.stack([_ids(11, 30, OC.END), _ids(12, 9, OC.END)])
    ids_g = np.stack([_ids(11, 30, 0), _ids(12, 9, 0)])
    weights = np.ones((2, 77), np.float32)
    weights[0, 3:7] = 1.3
    weights[1, 2:5] = 0.7
    ctx, pooled = mkimage.prompt_embeddings(L, G, ids_l, ids_g, weights)
    WL, WG = L.weights(), G.weights()
    plain, _ = mkimage.prompt_embeddings(L, G, ids_l, ids_g)
    L.close()
    G.close()
    ref, ref_p = OC.prompt_embeddings(_ocfg(cl), WL, _ocfg(cg), WG, ids_l, ids_g, weights)
    assert ctx.shape == (154, 640)
    assert _rel(ctx, ref) < 5e-3 and _cos(ctx, ref) >= 0.9999, (_rel(ctx, ref), _cos(ctx, ref))
    assert _rel(pooled, ref_p) < 5e-3
    # Unweighted tokens are the encoders' own states; weighted ones moved.
    assert np.array_equal(ctx[:3], plain[:3]) and not np.allclose(ctx[3:7], plain[3:7])


# Our weight -> the checkpoint's names (restated from Sdxl::load_clip, sdxl.cpp:154-237, independently of the loader).
def _ckpt(which, name):
    if name in ("tok", "pos"):
        return [("embeddings.token_embedding.weight" if name == "tok" else "embeddings.position_embedding.weight")
                if which == 0 else ("token_embedding.weight" if name == "tok" else "positional_embedding")]
    if name == "proj":
        return ["text_projection"]
    if name.startswith("lnf."):
        return ["ln_final.weight" if name.endswith(".w") else "ln_final.bias"]
    layer, part, wb = name.split(".")
    i = int(layer[1:])
    suf = ".weight" if wb == "w" else ".bias"
    if which == 0:
        pre = f"encoder.layers.{i}."
        if part == "qkv":
            return [pre + f"self_attn.{x}_proj" + suf for x in "qkv"]
        return [pre + {"ln1": "layer_norm1", "o": "self_attn.out_proj", "ln2": "layer_norm2", "fc1": "mlp.fc1",
                       "fc2": "mlp.fc2"}[part] + suf]
    pre = f"transformer.resblocks.{i}."
    if part == "qkv":
        return [pre + ("attn.in_proj_weight" if wb == "w" else "attn.in_proj_bias")]
    return [pre + {"ln1": "ln_1", "o": "attn.out_proj", "ln2": "ln_2", "fc1": "mlp.c_fc", "fc2": "mlp.c_proj"}[part]
            + suf]


@pytest.mark.parametrize("which", [0, 1])
def test_clip_checkpoint_names(cuda, tmp_path, which):
    import mkimage

    cfg = mkimage.ClipConfig(which=which, width=256, heads=4, layers=2, ffn=512, max_chunks=1)
    src = _model(mkimage, cfg, 61 + which)
    W = src.weights()
    src.close()
    prefix = "conditioner.embedders.0.transformer.text_model." if which == 0 else "conditioner.embedders.1.model."
    tensors = {}
    for name, a in W.items():
        parts = _ckpt(which, name)
        rows = a.shape[0] // len(parts)
        for k, n in enumerate(parts):
            bf16 = a.ndim == 2 and name not in ("tok", "pos", "proj")  # the bf16 matrices round-trip exactly
            tensors[prefix + n] = (a[k * rows:(k + 1) * rows], "BF16" if bf16 else "F32")
    tensors["model.diffusion_model.out.2.weight"] = (np.ones(8, np.float32), "F32")  # the UNet's: ignored
    p = tmp_path / "sdxl.safetensors"
    write_safetensors(p, tensors)
    dst = mkimage.Clip(cfg)
    assert dst.load_safetensors(p) == len(W)
    got = dst.weights()
    dst.close()
    for n, a in W.items():
        assert np.array_equal(got[n], a), n


def test_clip_rejects_bad_ids(cuda):
    import mkimage

    c = mkimage.Clip(mkimage.ClipConfig(which=1, width=256, heads=4, layers=2, ffn=512, max_chunks=1))
    c.init_random(3)
    ids = _ids(2, 5, 0)
    bad = ids.copy()
    bad[4] = 49408
    with pytest.raises(mkimage.MkbError, match="out of range"):
        c.encode(bad[None])
    no_end = ids.copy()
    no_end[no_end == OC.END] = 1
    with pytest.raises(mkimage.MkbError, match="end token"):
        c.encode(no_end[None])
    with pytest.raises(mkimage.MkbError):
        c.encode(np.stack([ids, ids]))  # more chunks than the handle takes
    h, p = c.encode(ids[None])  # the handle still works
    assert np.isfinite(h).all() and np.isfinite(p).all()
    c.close()
