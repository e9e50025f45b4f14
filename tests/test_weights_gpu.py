"""Checkpoint loading (mkb_dit_load_safetensors) and LoRA merges (mkb_dit_lora_merge / mkb_dit_load_lora) on the
device, both variants.

A synthetic checkpoint under each variant's tensor names (mixed F32 / BF16 / F16) is loaded strictly and every
weight read back must equal the expected values: bf16-rounded matrices, q/k/v and gate/up rows stacked in the
reference's order (qwen_image.cpp:79-111), the zero-centred text norm + 1. LoRA merges must equal the numpy oracle
(oracle.ops.lora_merge) on exactly the module's rows (qwen_image.cpp:295-331) within one bf16 rounding step, and
leave every other row untouched."""

import os
import sys

import numpy as np
import pytest

from oracle import ops as O

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from st_files import bf16_value, write_safetensors  # noqa: E402

pytestmark = pytest.mark.gpu

D, H, F, TD, NB = 256, 2, 512, 256, 2


def _cfg(variant):
    import mkimage

    return mkimage.DitConfig(variant=variant, hidden=D, heads=H, ffn=F, blocks=NB, text_dim=TD, max_batch=2,
                             max_text_tokens=32, max_image_tokens=64, slots=2)


def _ref21_ckpt(rng):
    r = lambda *s: rng.standard_normal(s).astype(np.float32) * 0.05  # noqa: E731
    ck = {"img_in.weight": r(D, 64), "txt_in.text_norm.weight": r(TD), "txt_in.in_layer.weight": r(D, TD),
          "txt_in.out_layer.weight": r(D, D), "time_text_embed.timestep_embedder.linear_1.weight": r(D, 256),
          "time_text_embed.timestep_embedder.linear_2.weight": r(D, D), "modulation.1.weight": r(4 * D, D),
          "norm_out.linear.weight": r(D, D), "proj_out.weight": r(64, D)}
    for i in range(NB):
        b = f"transformer_blocks.{i}."
        for n in ("attn.to_q", "attn.to_k", "attn.to_v", "attn.to_out.0"):
            ck[b + n + ".weight"] = r(D, D)
        ck[b + "attn.norm_q.weight"] = 1 + r(128)
        ck[b + "attn.norm_k.weight"] = 1 + r(128)
        ck[b + "img_mlp.gate_layer.weight"] = r(F, D)
        ck[b + "img_mlp.proj.weight"] = r(F, D)
        ck[b + "img_mlp.out.weight"] = r(D, F)
    return ck


def _ref21_expected(ck):
    m = lambda a: O.bf16_round(a)  # noqa: E731
    e = {"img_in.w": m(ck["img_in.weight"]), "txt_norm.w": ck["txt_in.text_norm.weight"] + 1.0,
         "txt_in1.w": m(ck["txt_in.in_layer.weight"]), "txt_in2.w": m(ck["txt_in.out_layer.weight"]),
         "time.lin1.w": m(ck["time_text_embed.timestep_embedder.linear_1.weight"]),
         "time.lin2.w": m(ck["time_text_embed.timestep_embedder.linear_2.weight"]),
         "mod.w": m(ck["modulation.1.weight"]), "norm_out.w": m(ck["norm_out.linear.weight"]),
         "proj_out.w": m(ck["proj_out.weight"])}
    for i in range(NB):
        b, p = f"transformer_blocks.{i}.", f"blk{i}."
        e[p + "qkv.w"] = m(np.concatenate([ck[b + f"attn.to_{x}.weight"] for x in "qkv"]))
        e[p + "o.w"] = m(ck[b + "attn.to_out.0.weight"])
        e[p + "norm_q"] = ck[b + "attn.norm_q.weight"]
        e[p + "norm_k"] = ck[b + "attn.norm_k.weight"]
        e[p + "gate_up.w"] = m(np.concatenate([ck[b + "img_mlp.gate_layer.weight"], ck[b + "img_mlp.proj.weight"]]))
        e[p + "down.w"] = m(ck[b + "img_mlp.out.weight"])
    return e


def _qwen1_ckpt(rng):
    r = lambda *s: rng.standard_normal(s).astype(np.float32) * 0.05  # noqa: E731
    ck = {}

    def lin(name, o, i):
        ck[name + ".weight"] = r(o, i)
        ck[name + ".bias"] = r(o)

    lin("img_in", D, 64)
    ck["txt_norm.weight"] = 1 + r(TD)
    lin("txt_in", D, TD)
    lin("time_text_embed.timestep_embedder.linear_1", D, 256)
    lin("time_text_embed.timestep_embedder.linear_2", D, D)
    lin("norm_out.linear", 2 * D, D)
    lin("proj_out", 64, D)
    for i in range(NB):
        b = f"transformer_blocks.{i}."
        lin(b + "img_mod.1", 6 * D, D)
        lin(b + "txt_mod.1", 6 * D, D)
        for n in ("to_q", "to_k", "to_v", "add_q_proj", "add_k_proj", "add_v_proj", "to_out.0", "to_add_out"):
            lin(b + "attn." + n, D, D)
        for n in ("norm_q", "norm_k", "norm_added_q", "norm_added_k"):
            ck[b + "attn." + n + ".weight"] = 1 + r(128)
        for s in ("img", "txt"):
            lin(b + s + "_mlp.net.0.proj", F, D)
            lin(b + s + "_mlp.net.2", D, F)
    return ck


def _qwen1_expected(ck):
    m = lambda a: O.bf16_round(a)  # noqa: E731
    e = {}

    def lin(ours, theirs):
        e[ours + ".w"] = m(ck[theirs + ".weight"])
        e[ours + ".b"] = ck[theirs + ".bias"]

    lin("img_in", "img_in")
    e["txt_norm.w"] = ck["txt_norm.weight"]
    lin("txt_in", "txt_in")
    lin("time.lin1", "time_text_embed.timestep_embedder.linear_1")
    lin("time.lin2", "time_text_embed.timestep_embedder.linear_2")
    lin("norm_out", "norm_out.linear")
    lin("proj_out", "proj_out")
    for i in range(NB):
        b, p = f"transformer_blocks.{i}.", f"blk{i}."
        for s, q, k, v, o, nq, nk in (("img", "to_q", "to_k", "to_v", "to_out.0", "norm_q", "norm_k"),
                                      ("txt", "add_q_proj", "add_k_proj", "add_v_proj", "to_add_out", "norm_added_q",
                                       "norm_added_k")):
            lin(p + s + ".mod", b + s + "_mod.1")
            e[p + s + ".qkv.w"] = m(np.concatenate([ck[b + "attn." + x + ".weight"] for x in (q, k, v)]))
            e[p + s + ".qkv.b"] = np.concatenate([ck[b + "attn." + x + ".bias"] for x in (q, k, v)])
            lin(p + s + ".o", b + "attn." + o)
            e[p + s + ".norm_q"] = ck[b + "attn." + nq + ".weight"]
            e[p + s + ".norm_k"] = ck[b + "attn." + nk + ".weight"]
            lin(p + s + ".ff1", b + s + "_mlp.net.0.proj")
            lin(p + s + ".ff2", b + s + "_mlp.net.2")
    return e


def _dtypes(ck):
    """Block-0 matrices stored as BF16, block-1 norms as F16, the rest F32; values made exact in those types."""
    dt = {}
    for n, a in ck.items():
        if a.ndim == 2 and "transformer_blocks.0." in n:
            ck[n] = bf16_value(a).reshape(a.shape)
            dt[n] = "BF16"
        elif a.ndim == 1 and "transformer_blocks.1." in n and "norm" in n:
            ck[n] = a.astype(np.float16).astype(np.float32)
            dt[n] = "F16"
        else:
            dt[n] = "F32"
    return dt


def _write_shards(tmp_path, ck, dt):
    names = sorted(ck)
    half = len(names) // 2
    paths = [tmp_path / "part-00001.safetensors", tmp_path / "part-00002.safetensors"]
    write_safetensors(paths[0], {n: (ck[n], dt[n]) for n in names[:half]}, metadata={"format": "pt"})
    write_safetensors(paths[1], {n: (ck[n], dt[n]) for n in names[half:]})
    return paths


def _model(variant, seed, tmp_path):
    import mkimage

    rng = np.random.RandomState(seed)
    ck = _ref21_ckpt(rng) if variant == "ref21" else _qwen1_ckpt(rng)
    dt = _dtypes(ck)
    d = mkimage.Dit(_cfg(mkimage.REF21 if variant == "ref21" else mkimage.QWEN1))
    n = d.load_safetensors(_write_shards(tmp_path, ck, dt), strict=True)
    return d, ck, n


@pytest.mark.parametrize("variant", ["ref21", "qwen1"])
def test_load_checkpoint(cuda, tmp_path, variant):
    d, ck, n = _model(variant, 11, tmp_path)
    assert n == len(ck)
    exp = _ref21_expected(ck) if variant == "ref21" else _qwen1_expected(ck)
    got = d.weights()
    assert set(got) == set(exp)
    for k, want in exp.items():
        assert np.array_equal(got[k], want.reshape(got[k].shape)), k


def test_load_errors(cuda, tmp_path):
    import mkimage

    ck = _ref21_ckpt(np.random.RandomState(5))
    d = mkimage.Dit(_cfg(mkimage.REF21))
    p = tmp_path / "c.safetensors"
    bad = dict(ck)
    bad["transformer_blocks.0.attn.to_q.weight"] = np.zeros((D, D + 8), np.float32)
    write_safetensors(p, bad)
    with pytest.raises(mkimage.MkbError, match="needs"):
        d.load_safetensors(p)
    miss = dict(ck)
    del miss["proj_out.weight"]
    write_safetensors(p, miss)
    with pytest.raises(mkimage.MkbError, match="unwritten"):
        d.load_safetensors(p)
    extra = dict(ck)
    extra["transformer_blocks.7.attn.to_q.weight"] = np.zeros((D, D), np.float32)  # a block the model lacks
    write_safetensors(p, extra)
    with pytest.raises(mkimage.MkbError, match="matches no weight"):
        d.load_safetensors(p)
    assert d.load_safetensors(p, strict=False) == len(ck)


def _merged_ok(got, W, A, B, s):
    """The device merge within one bf16 step of the oracle (2^-7 relative, the device sums in fp32 and rounds once,
    the oracle in float64 and rounds twice, so the two can straddle a rounding tie), measured against the operands'
    size: where W and s B A nearly cancel, a fixed rounding difference is many steps of the small result."""
    want = O.lora_merge(W, A, B, s)
    delta = s * (B.astype(np.float64) @ A.astype(np.float64))
    return bool(np.all(np.abs(got - want) <= 2.0 ** -7 * (np.abs(W) + np.abs(delta)) + 1e-30))


def test_lora_file_ref21(cuda, tmp_path):
    d, _, _ = _model("ref21", 12, tmp_path)
    before = d.weights()
    rng = np.random.RandomState(13)
    r, scale = 8, 0.7
    # module -> (weight, first row, rows, in features, alpha)
    mods = {"transformer_blocks.0.attn.to_k": ("blk0.qkv.w", D, D, D, None),
            "transformer_blocks.1.img_mlp.gate_layer": ("blk1.gate_up.w", 0, F, D, 16.0),
            "transformer_blocks.1.img_mlp.proj": ("blk1.gate_up.w", F, F, D, None),
            "modulation.1": ("mod.w", 0, 4 * D, D, 4.0)}
    tensors, pairs = {}, {}
    for m, (w, r0, rows, cin, alpha) in mods.items():
        A = rng.standard_normal((r, cin)).astype(np.float32) * 0.1
        B = rng.standard_normal((rows, r)).astype(np.float32) * 0.1
        tensors["transformer." + m + ".lora_A.weight"] = A
        tensors["transformer." + m + ".lora_B.weight"] = B
        if alpha is not None:
            tensors["transformer." + m + ".alpha"] = np.array(alpha, np.float32)
        pairs[m] = (A, B, alpha)
    p = tmp_path / "lora.safetensors"
    write_safetensors(p, tensors)
    assert d.load_lora(p, scale) == len(mods)
    after = d.weights()
    touched = {}
    for m, (w, r0, rows, _, _) in mods.items():
        A, B, alpha = pairs[m]
        s = scale * (alpha / r if alpha is not None else 1.0)
        assert _merged_ok(after[w][r0:r0 + rows], before[w][r0:r0 + rows], A, B, s), m
        touched.setdefault(w, []).append((r0, rows))
    for w, a in before.items():
        mask = np.ones(a.shape[0], bool)
        for r0, rows in touched.get(w, []):
            mask[r0:r0 + rows] = False
        assert np.array_equal(after[w][mask], a[mask]), w


def test_lora_merge_qwen1_and_errors(cuda, tmp_path):
    import mkimage

    d, _, _ = _model("qwen1", 14, tmp_path)
    before = d.weights()
    rng = np.random.RandomState(15)
    A = rng.standard_normal((4, D)).astype(np.float32) * 0.1
    B = rng.standard_normal((D, 4)).astype(np.float32) * 0.1
    d.lora_merge("transformer_blocks.1.attn.add_v_proj", A, B, 1.5)  # text stream, v rows of the stacked qkv
    A2 = rng.standard_normal((16, F)).astype(np.float32) * 0.05
    B2 = rng.standard_normal((D, 16)).astype(np.float32) * 0.05
    d.lora_merge("transformer_blocks.0.img_mlp.net.2", A2, B2, 1.0)
    after = d.weights()
    w = "blk1.txt.qkv.w"
    assert _merged_ok(after[w][2 * D:], before[w][2 * D:], A, B, 1.5)
    assert np.array_equal(after[w][:2 * D], before[w][:2 * D])
    w = "blk0.img.ff2.w"
    assert _merged_ok(after[w], before[w], A2, B2, 1.0)
    assert np.array_equal(after["blk0.txt.ff2.w"], before["blk0.txt.ff2.w"])
    with pytest.raises(mkimage.MkbError, match="adapter"):  # D inputs where the module takes F
        d.lora_merge("transformer_blocks.0.img_mlp.net.2", A2[:, :D].copy(), B2, 1.0)
    with pytest.raises(ValueError):
        d.lora_merge("transformer_blocks.0.img_mlp.net.2", A2, B, 1.0)  # B's rank (4) is not A's (16)
    with pytest.raises(mkimage.MkbError, match="not a matrix"):
        d.lora_merge("transformer_blocks.0.attn.nope", A, B, 1.0)
    assert mkimage.ops.check_kernels() == 0
