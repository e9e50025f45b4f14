"""SDXL UNet and VAE checkpoints (mkb_unet_load_safetensors / mkb_vae_load_safetensors) by the reference's tensor
names: a randomly initialised model's weights written out under the checkpoint names (restated here independently
of the loader from sdxl.cpp:238-362 and engine.cpp:92-118, 590-640: convolutions as [out][in][ky][kx], stacked q/k/v
and cross k/v split, 1x1 convolutions 4-D) must load into a fresh model exactly, with unrelated tensors (a
single-file checkpoint's text encoders) ignored and a missing tensor an error under strict loading."""

import os
import re
import sys

import numpy as np
import pytest

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from st_files import write_safetensors  # noqa: E402

pytestmark = pytest.mark.gpu

RES = {"gn1": "in_layers.0", "conv1": "in_layers.2", "gn2": "out_layers.0", "conv2": "out_layers.3",
       "skip": "skip_connection", "emb": "emb_layers.1"}
TB = {"ln1": "norm1", "ln2": "norm2", "ln3": "norm3", "o1": "attn1.to_out.0", "q2": "attn2.to_q",
      "o2": "attn2.to_out.0", "ff1": "ff.net.0.proj", "ff2": "ff.net.2"}


def _wb(s):
    return ".weight" if s == "w" else ".bias"


def _ckpt_value(a):
    """Table layout -> checkpoint layout: a 3x3 convolution [o][3][3][i] -> [o][i][3][3]."""
    return a.transpose(0, 3, 1, 2).copy() if a.ndim == 4 else a


def unet_names(name, all_names):
    """Our UNet weight -> [(checkpoint name, rows)] (rows None: the whole tensor)."""
    m = re.fullmatch(r"(conv_in|time\.lin1|time\.lin2|label\.lin1|label\.lin2|out\.gn|out\.conv)\.([wb])", name)
    if m:
        top = {"conv_in": "input_blocks.0.0", "time.lin1": "time_embed.0", "time.lin2": "time_embed.2",
               "label.lin1": "label_emb.0.0", "label.lin2": "label_emb.0.2", "out.gn": "out.0", "out.conv": "out.2"}
        return [(top[m[1]] + _wb(m[2]), None)]
    m = re.fullmatch(r"(in|out)(\d+)\.(.*)", name) or re.fullmatch(r"(mid)\.(res0|attn|res1)\.(.*)", name)
    if m[1] == "mid":
        blk = "middle_block."
        idx = {"res0": "0", "attn": "1", "res1": "2"}[m[2]]
        kind, rest = ("res" if m[2].startswith("res") else "attn"), m[3]
    else:
        blk = ("input_blocks." if m[1] == "in" else "output_blocks.") + m[2] + "."
        kind, rest = m[3].split(".", 1)
        idx = {"res": "0", "attn": "1", "down": "0", "up": None}[kind]
    if kind == "down":
        return [(blk + "0.op" + _wb(rest), None)]
    if kind == "up":
        has_attn = any(n.startswith(f"{m[1]}{m[2]}.attn.") for n in all_names)
        return [(blk + ("2" if has_attn else "1") + ".conv" + _wb(rest), None)]
    stem, s = rest.rsplit(".", 1)
    base = blk + idx + "."
    if kind == "res":
        return [(base + RES[stem] + _wb(s), None)]
    if stem in ("gn", "proj_in", "proj_out"):
        return [(base + {"gn": "norm"}.get(stem, stem) + _wb(s), None)]
    j, what = re.fullmatch(r"b(\d+)\.(\w+)", stem).groups()
    tb = f"{base}transformer_blocks.{j}."
    if what == "qkv":
        return [(tb + f"attn1.to_{x}" + _wb(s), 1 / 3) for x in "qkv"]
    if what == "kv2":
        return [(tb + f"attn2.to_{x}" + _wb(s), 1 / 2) for x in "kv"]
    return [(tb + TB[what] + _wb(s), None)]


def vae_names(name, ldm):
    """Our VAE weight -> [(checkpoint name, rows)], Diffusers or original AutoencoderKL names."""
    stem, s = name.rsplit(".", 1)
    w = _wb(s)
    top = {"post_quant": ("post_quant_conv", "post_quant_conv"), "conv_in": ("decoder.conv_in", "decoder.conv_in"),
           "out.gn": ("decoder.conv_norm_out", "decoder.norm_out"), "out.conv": ("decoder.conv_out", "decoder.conv_out"),
           "mid.attn.gn": ("decoder.mid_block.attentions.0.group_norm", "decoder.mid.attn_1.norm"),
           "mid.attn.proj": ("decoder.mid_block.attentions.0.to_out.0", "decoder.mid.attn_1.proj_out")}
    if stem in top:
        return [(top[stem][ldm] + w, None)]
    if stem == "mid.attn.qkv":
        pre = "decoder.mid.attn_1." if ldm else "decoder.mid_block.attentions.0.to_"
        return [(pre + x + w, 1 / 3) for x in "qkv"]
    res = {"gn1": "norm1", "conv1": "conv1", "gn2": "norm2", "conv2": "conv2",
           "skip": "nin_shortcut" if ldm else "conv_shortcut"}
    m = re.fullmatch(r"mid\.res(\d)\.(\w+)", stem)
    if m:
        k = int(m[1])
        return [((f"decoder.mid.block_{k + 1}." if ldm else f"decoder.mid_block.resnets.{k}.") + res[m[2]] + w, None)]
    m = re.fullmatch(r"up(\d)\.res(\d)\.(\w+)", stem)
    if m:
        i, k = int(m[1]), int(m[2])
        return [((f"decoder.up.{3 - i}.block.{k}." if ldm else f"decoder.up_blocks.{i}.resnets.{k}.") + res[m[3]] + w,
                 None)]
    m = re.fullmatch(r"up(\d)\.up", stem)
    i = int(m[1])
    return [((f"decoder.up.{3 - i}.upsample.conv" if ldm else f"decoder.up_blocks.{i}.upsamplers.0.conv") + w, None)]


def _write(path, weights, mapping, prefix, one_by_one):
    tensors = {}
    for name, a in weights.items():
        parts = mapping(name)
        if len(parts) == 1:
            v = _ckpt_value(a)
            if one_by_one(name) and v.ndim == 2:
                v = v[:, :, None, None]  # a 1x1 convolution
            tensors[prefix + parts[0][0]] = (v, "BF16" if v.ndim > 1 and len(tensors) % 2 else "F32")
        else:
            for k, (n, _) in enumerate(parts):
                rows = a.shape[0] // len(parts)
                tensors[prefix + n] = (a[k * rows:(k + 1) * rows], "F32")
    tensors["conditioner.embedders.0.transformer.text_model.final_layer_norm.weight"] = (np.ones(8, np.float32), "F32")
    write_safetensors(path, tensors)
    return tensors


def test_unet_checkpoint_round_trip(cuda, tmp_path):
    import mkimage

    cfg = mkimage.UnetConfig(channels=(64, 128, 128), depth=(0, 1, 1), layers=1, context_dim=64, pooled_dim=64,
                             max_batch=2, max_gh=8, max_gw=8, max_context=8, slots=2)
    src = mkimage.Unet(cfg)
    src.init_random(seed=21)
    W = src.weights()
    names = list(W)
    p = tmp_path / "unet.safetensors"
    tensors = _write(p, W, lambda n: unet_names(n, names), "model.diffusion_model.", lambda n: n.endswith("skip.w"))
    dst = mkimage.Unet(cfg)
    assert dst.load_safetensors(p) == len(W)
    got = dst.weights()
    for n, a in W.items():
        assert np.array_equal(got[n], a), n
    missing = dict(tensors)
    del missing["model.diffusion_model.out.2.weight"]
    write_safetensors(p, missing)
    with pytest.raises(mkimage.MkbError, match="lack"):
        mkimage.Unet(cfg).load_safetensors(p)
    assert mkimage.Unet(cfg).load_safetensors(p, strict=False) == len(W) - 1


@pytest.mark.parametrize("ldm", [False, True])
def test_vae_checkpoint_round_trip(cuda, tmp_path, ldm):
    import mkimage

    cfg = mkimage.VaeConfig(channels=(128, 128, 256, 256), layers=1, max_gh=8, max_gw=8)
    src = mkimage.Vae(cfg)
    src.init_random(seed=22)
    W = src.weights()
    p = tmp_path / "vae.safetensors"
    one = (lambda n: n.startswith(("post_quant", "mid.attn.")) or n.endswith("skip.w")) if ldm else \
        (lambda n: n.startswith("post_quant") or n.endswith("skip.w"))
    _write(p, W, lambda n: vae_names(n, ldm), "first_stage_model." if ldm else "", one)
    dst = mkimage.Vae(cfg)
    assert dst.load_safetensors(p) == len(W)
    got = dst.weights()
    for n, a in W.items():
        assert np.array_equal(got[n], a), n


def test_unet_lora(cuda, tmp_path):
    """LoRA on the UNet's transformer projections (sdxl.cpp:385-417) against oracle.ops.lora_merge: a kohya-style
    flattened module name with alpha, a PEFT-style name on the GEGLU projection (interleaved rows), a direct merge;
    every other row untouched."""
    import mkimage
    from oracle import ops as O

    cfg = mkimage.UnetConfig(channels=(64, 128, 128), depth=(0, 1, 1), layers=1, context_dim=64, pooled_dim=64,
                             max_batch=2, max_gh=8, max_gw=8, max_context=8, slots=2)
    u = mkimage.Unet(cfg)
    u.init_random(seed=23)
    before = u.weights()
    rng = np.random.RandomState(24)
    c = 128
    r = 8
    A1, B1 = rng.standard_normal((r, c)).astype(np.float32) * 0.1, rng.standard_normal((c, r)).astype(np.float32) * 0.1
    A2 = rng.standard_normal((r, c)).astype(np.float32) * 0.1
    B2 = rng.standard_normal((8 * c, r)).astype(np.float32) * 0.1
    p = tmp_path / "lora.safetensors"
    write_safetensors(p, {"lora_unet_input_blocks_3_1_transformer_blocks_0_attn1_to_k.lora_down.weight": A1,
                          "lora_unet_input_blocks_3_1_transformer_blocks_0_attn1_to_k.lora_up.weight": B1,
                          "lora_unet_input_blocks_3_1_transformer_blocks_0_attn1_to_k.alpha": np.array(4.0, np.float32),
                          "input_blocks.3.1.transformer_blocks.0.ff.net.0.proj.lora_A.weight": A2,
                          "input_blocks.3.1.transformer_blocks.0.ff.net.0.proj.lora_B.weight": B2})
    assert u.load_lora(p, 0.8) == 2
    A3 = rng.standard_normal((4, 64)).astype(np.float32) * 0.1  # cross-attention reads 64-wide context
    B3 = rng.standard_normal((c, 4)).astype(np.float32) * 0.1
    u.lora_merge("middle_block.1.transformer_blocks.0.attn2.to_v", A3, B3, 1.2)
    after = u.weights()

    def ok(got, W, A, B, s):
        want = O.lora_merge(W, A, B, s)
        delta = s * (B.astype(np.float64) @ A.astype(np.float64))
        return bool(np.all(np.abs(got - want) <= 2.0 ** -7 * (np.abs(W) + np.abs(delta)) + 1e-30))

    changed = {"in3.attn.b0.qkv.w": (c, 2 * c), "in3.attn.b0.ff1.w": (0, 8 * c), "mid.attn.b0.kv2.w": (c, 2 * c)}
    q = "in3.attn.b0.qkv.w"
    assert ok(after[q][c:2 * c], before[q][c:2 * c], A1, B1, 0.8 * 4.0 / r)
    f = "in3.attn.b0.ff1.w"
    assert ok(after[f], before[f], A2, B2, 0.8)
    k = "mid.attn.b0.kv2.w"
    assert ok(after[k][c:], before[k][c:], A3, B3, 1.2)
    for n, a in before.items():
        mask = np.ones(a.shape[0], bool)
        if n in changed:
            mask[changed[n][0]:changed[n][1]] = False
        assert np.array_equal(after[n][mask], a[mask]), n
    with pytest.raises(mkimage.MkbError, match="not a projection"):
        u.lora_merge("input_blocks.1.0.in_layers.2", A1, B1, 1.0)
