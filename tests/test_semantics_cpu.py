"""Sensitivity of the parity tests to each semantic choice the oracle had to infer.

The reference's GEMM, attention and per-head norm kernels live in its absent runtime, so a few of the oracle's
choices are inferred from call sites rather than read from code: per-head RMSNorm before RoPE, RoPE on interleaved
pairs (mode 2), SwiGLU as silu(first half) x second half, the condition-causal mask of the reference variant (text
rows causal among themselves, never seeing an image key), the text rows' modulation row (t = 0) and its
tanh-squashed gates. The device kernels implement the same choices, so
the GPU parity tests cannot tell whether a choice is right; what they can do is notice a kernel that made the other
choice. Each test here flips one choice in the oracle alone and checks that what the first block adds to the
residual stream (its output minus its input) moves beyond the tolerance the GPU tests hold that contribution to
(cosine >= 0.999): a kernel with the flipped choice would fail them. The contribution, not the block output, is
the sensitive quantity: with weights of scale 0.02 the residual carried through a block dwarfs what it adds."""

import numpy as np
import pytest

from oracle import ops as O
from oracle import qwen_dit as QD
from oracle import rng


def _weights(cfg, seed):
    """Random weights with an O(1) modulation: the time MLP and modulation matrices scaled (STRONG_MOD) so gates,
    scales and shifts are of order one, as in a trained model; at the 0.02 scale of every other matrix they are
    ~0.01, where tanh(g) and g or (1 + scale) and 1 cannot be told apart. Norm weights 1 + 0.5 N(0, 1)."""
    W = {}
    for i, (name, shape) in enumerate(QD.weight_shapes(cfg).items()):
        a = rng.normal(rng.tensor_key(seed, i), int(np.prod(shape))).reshape(shape)
        if name.startswith("txt_norm") or name.endswith(("norm_q", "norm_k")):
            W[name] = (1.0 + 0.5 * a).astype(np.float32)
        else:
            sd = 0.02 * STRONG_MOD.get(name.split(".", 1)[-1] if name.startswith("blk") else name, 1.0)
            W[name] = O.bf16_round(sd * a) if len(shape) == 2 else (sd * a).astype(np.float32)
    return W


# Scale factors over the 0.02 init that give the modulation path O(1) outputs (D = 256 here and in the GPU tests'
# strong-modulation cases): keys are weight names, block prefixes dropped.
STRONG_MOD = {"time.lin1.w": 4.0, "time.lin2.w": 6.0, "mod.w": 12.0, "txt.mod.w": 12.0, "img.mod.w": 12.0,
              "norm_out.w": 12.0}


def _case(variant):
    cfg = QD.default_cfg(variant, D=256, heads=2, F=512, blocks=2, text_dim=128)
    W = _weights(cfg, 41 if variant == "qwen1" else 43)
    S, h, w = 9, 6, 7
    prompt = rng.normal(rng.tensor_key(44, 0), S * 128).reshape(S, 128)
    lat = rng.normal(rng.tensor_key(44, 1), h * w * 64).reshape(h * w, 64)
    return cfg, W, prompt, lat, h, w


def _moved(a, b):
    """True when b is outside the GPU parity tests' tolerance on a block's contribution (cosine >= 0.999)."""
    a64, b64 = a.astype(np.float64).ravel(), b.astype(np.float64).ravel()
    cos = a64 @ b64 / np.sqrt((a64 @ a64) * (b64 @ b64))
    return cos < 0.999, cos


def _run(variant):
    """Block 0's contribution on the first step: its output rows minus its input rows (text then image)."""
    cfg, W, prompt, lat, h, w = _case(variant)
    got = {}
    QD.step(cfg, W, lat, prompt, 0.6, h, w, state={} if variant == "ref21" else None,
            probe=lambda name, a: got.__setitem__(name, a))
    return got["block0"] - np.concatenate([got["txt_in"], got["img_in"]])


def _flipped(monkeypatch, variant, target, attr, fn):
    base = _run(variant)
    monkeypatch.setattr(target, attr, fn)
    moved, stats = _moved(base, _run(variant))
    assert moved, stats


@pytest.mark.parametrize("variant", ["qwen1", "ref21"])
def test_rope_after_norm(monkeypatch, variant):
    """RoPE applied before the per-head RMSNorm (the norm's per-dimension weight does not commute with rotation)."""
    rms, rope = O.rms_norm, O.rope_pairs
    pending = {}

    def norm_later(x, w, eps=1e-6):
        if x.ndim == 3 and x.shape[-1] == QD.HEAD_DIM:  # per-head q / k norm: defer it past the rotation
            pending["w"], pending["eps"] = w, eps
            return x
        return rms(x, w, eps)

    def rope_then_norm(x, cs):
        return rms(rope(x, cs), pending.pop("w"), pending.pop("eps"))

    base = _run(variant)
    monkeypatch.setattr(O, "rms_norm", norm_later)
    monkeypatch.setattr(O, "rope_pairs", rope_then_norm)
    moved, stats = _moved(base, _run(variant))
    assert moved, stats


@pytest.mark.parametrize("variant", ["qwen1", "ref21"])
def test_rope_half_split_pairs(monkeypatch, variant):
    """RoPE on (x[i], x[i + 64]) pairs instead of the interleaved (x[2i], x[2i + 1])."""

    def half_split(x, cs):
        x = np.asarray(x, np.float32)
        x0, x1 = x[..., :64], x[..., 64:]
        c, s = cs[..., 0], cs[..., 1]
        return np.concatenate([x0 * c - x1 * s, x0 * s + x1 * c], axis=-1)

    _flipped(monkeypatch, variant, O, "rope_pairs", half_split)


def test_swiglu_halves_swapped(monkeypatch):
    """SwiGLU as silu(second half) x first half."""
    cfg = _case("ref21")[0]
    F = cfg["F"]
    base = _run("ref21")

    def block_swapped(cfg_, W, i, x, split, mod, rope, kv_cache=None):
        Wi = dict(W)
        gu = W[f"blk{i}.gate_up.w"]
        Wi[f"blk{i}.gate_up.w"] = np.concatenate([gu[F:], gu[:F]])  # the kernel reading the halves the other way
        return orig(cfg_, Wi, i, x, split, mod, rope, kv_cache)

    orig = QD.block_ref21
    monkeypatch.setattr(QD, "block_ref21", block_swapped)
    moved, stats = _moved(base, _run("ref21"))
    assert moved, stats


def test_ref21_fully_joint_mask(monkeypatch):
    """The reference variant with text rows attending to image keys too (no condition-causal mask)."""
    att = O.attention
    _flipped(monkeypatch, "ref21", O, "attention", lambda q, k, v, mask=None: att(q, k, v, None))


def test_ref21_text_rows_see_every_text_key(monkeypatch):
    """The reference variant with its text rows attending to all text keys (the runtime's `block` argument cutting
    off only the image keys) instead of causally to keys 0..p."""
    att = O.attention

    def all_text(q, k, v, mask=None):
        if mask is not None:
            text = ~mask.all(axis=1)  # the text rows: the only rows that do not see every key
            mask = mask.copy()
            mask[np.ix_(text, np.arange(int(text.sum())))] = True
        return att(q, k, v, mask)

    _flipped(monkeypatch, "ref21", O, "attention", all_text)


def test_ref21_text_rows_take_the_image_modulation(monkeypatch):
    """Text rows modulated by row 0 (sigma) instead of row 1 (t = 0): all rows the image's modulation."""
    lin = O.linear

    def same_rows(x, w, b=None):
        y = lin(x, w, b)
        if y.ndim == 2 and y.shape[0] == 2 and w.shape[0] == 4 * 256:  # the shared modulation's two rows
            y = np.stack([y[0], y[0]])
        return y

    _flipped(monkeypatch, "ref21", O, "linear", same_rows)


class _NumpyWithoutTanh:
    """numpy as the oracle's block code sees it, with tanh the identity (the gates only: the GELU of the text input
    uses the ops module's own reference to numpy)."""

    tanh = staticmethod(lambda a: np.asarray(a))

    def __getattr__(self, name):
        return getattr(np, name)


def test_ref21_plain_gates(monkeypatch):
    """x += g * y instead of x += tanh(g) * y."""
    _flipped(monkeypatch, "ref21", QD, "np", _NumpyWithoutTanh())


def test_ref21_text_cache_second_step_matches_full_rerun():
    """The text K/V cache is exact: a second step with the cache equals recomputing the text rows (text rows never
    see image keys, so their K/V do not change between steps)."""
    cfg, W, prompt, lat, h, w = _case("ref21")
    state = {}
    QD.step(cfg, W, lat, prompt, 0.6, h, w, state=state)
    cached = QD.step(cfg, W, lat, prompt, 0.5, h, w, state=state)
    full = QD.step(cfg, W, lat, prompt, 0.5, h, w, state=None)
    assert np.allclose(cached, full, atol=1e-5, rtol=1e-5)


def test_modulation_is_order_one():
    """The strong-modulation weights above put the gates in the range where their form matters."""
    for variant in ("qwen1", "ref21"):
        cfg, W, prompt, lat, h, w = _case(variant)
        st = O.silu(QD.time_embedding(W, 0.6))
        name = "mod.w" if variant == "ref21" else "blk0.img.mod.w"
        mod = O.linear(st[None], W[name], W.get(name[:-1] + "b"))[0]
        rms = float(np.sqrt((mod.astype(np.float64) ** 2).mean()))
        assert 0.3 < rms < 5.0, (variant, rms)
