"""Parity of the denoiser step (mkb_dit_*) against the numpy oracle on identical seeded inputs.

Bar (per block output, the north star's): max-abs <= 2e-2 and cosine >= 0.999; final velocities: the reference's
own relative RMS < 0.05 (tests/image_ref_test.cpp:146) plus the same cosine. Weights are generated on the device
by seed and read back for the oracle; prompts and latents are generated on the host (oracle/rng.py)."""

import numpy as np
import pytest

from oracle import qwen_dit as QD
from oracle import rng

pytestmark = pytest.mark.gpu

MAX_ABS, MIN_COS, MAX_REL = 2e-2, 0.999, 0.05


def _cos(a, b):
    a, b = a.astype(np.float64).ravel(), b.astype(np.float64).ravel()
    return float(a @ b / np.sqrt((a @ a) * (b @ b)))


def _row_cos_min(a, b, width):
    a = a.reshape(-1, width).astype(np.float64)
    b = b.reshape(-1, width).astype(np.float64)
    return float(((a * b).sum(1) / np.sqrt((a * a).sum(1) * (b * b).sum(1))).min())


def _rel(got, want):
    return float(np.sqrt(((got.astype(np.float64) - want) ** 2).sum() / (want.astype(np.float64) ** 2).sum()))


def _make(variant, D, H, F, blocks, TD, B, S, N, seed=7):
    import mkimage

    cfg = mkimage.DitConfig(variant=variant, hidden=D, heads=H, ffn=F, blocks=blocks, text_dim=TD, max_batch=B,
                            max_text_tokens=S, max_image_tokens=N, slots=max(2, B))
    d = mkimage.Dit(cfg)
    d.init_random(seed)
    return d, QD.default_cfg("qwen1" if variant == 0 else "ref21", D, H, F, blocks, TD)


def _inputs(B, S, N, TD, seed=11):
    prompts = [rng.normal(rng.tensor_key(seed, 100 + b), S * TD).reshape(S, TD) for b in range(B)]
    lats = [rng.normal(rng.tensor_key(seed, 200 + b), N * 64).reshape(N, 64) for b in range(B)]
    return prompts, lats


def _check_block(got, want, what):
    err = float(np.abs(got - want).max())
    cos = _cos(got, want)
    assert err <= MAX_ABS and cos >= MIN_COS, f"{what}: max-abs {err:.3e}, cosine {cos:.6f}"


def _check_delta(got_out, got_in, want_out, want_in, what):
    """What a block adds to the residual stream (output minus input) on both sides: the residual it carries through
    dominates its output, so this is the check that sees the block's own arithmetic."""
    cos = _cos(got_out - got_in, want_out - want_in)
    assert cos >= MIN_COS, f"{what}: contribution cosine {cos:.6f}"


@pytest.mark.parametrize("h,w,S,B", [(16, 16, 40, 2), (10, 13, 7, 1)])
def test_qwen1_blocks_and_velocity(cuda, h, w, S, B):
    """qwen1 at a reduced width (3 blocks): every block's text and image rows, then the velocity."""
    D, H, F, NB, TD = 512, 4, 1024, 3, 384
    N = h * w
    d, cfg = _make(0, D, H, F, NB, TD, B, S, N)
    W = d.weights()
    prompts, lats = _inputs(B, S, N, TD)
    sigmas = [0.5, 0.8][:B]
    for b in range(B):
        d.begin(prompts[b], h, w, slot=b)
    got = {}
    d.set_probe(lambda name, layer, a: got.__setitem__((name, layer), a))
    vel = d.step_batch(list(range(B)), np.stack(lats), sigmas)
    d.set_probe(None)
    for b in range(B):
        want = {}
        v_ref = QD.step(cfg, W, lats[b], prompts[b], sigmas[b], h, w,
                        probe=lambda name, a: want.__setitem__(name, a))
        prev = np.concatenate([got[("txt_in", -1)].reshape(B, S, D)[b], got[("img_in", -1)].reshape(B, N, D)[b]])
        prev_want = np.concatenate([want["txt_in"], want["img_in"]])
        for i in range(NB):
            gt = got[("block.txt", i)].reshape(B, S, D)[b]
            gi = got[("block.img", i)].reshape(B, N, D)[b]
            out = np.concatenate([gt, gi])
            _check_block(out, want[f"block{i}"], f"sample {b} block {i}")
            _check_delta(out, prev, want[f"block{i}"], prev_want, f"sample {b} block {i}")
            prev, prev_want = out, want[f"block{i}"]
        _check_block(got[("temb", -1)].reshape(B, D)[b], want["temb"], "temb")
        v = vel[b]
        assert _rel(v, v_ref) < MAX_REL and _cos(v, v_ref) >= MIN_COS
        assert np.abs(v - v_ref).max() <= MAX_ABS * max(1.0, np.abs(v_ref).max())


def test_ref21_two_steps_with_text_cache(cuda):
    """ref21 (the reference's own math): step 1 runs text + image rows and caches the text K/V per block; step 2
    runs the image rows only against the cache (qwen_image.cpp:152-158, 251-262)."""
    D, H, F, NB, TD = 512, 4, 768, 3, 512
    h, w, S, B = 12, 12, 33, 2
    N = h * w
    d, cfg = _make(1, D, H, F, NB, TD, B, S, N, seed=5)
    W = d.weights()
    prompts, lats = _inputs(B, S, N, TD, seed=3)
    for b in range(B):
        d.begin(prompts[b], h, w, slot=b)
    states = [dict() for _ in range(B)]
    for step_i, sig in enumerate([0.9, 0.6]):
        got = {}
        d.set_probe(lambda name, layer, a: got.__setitem__((name, layer), a))
        vel = d.step_batch([0, 1], np.stack(lats), [sig, sig])
        d.set_probe(None)
        T = S + N if step_i == 0 else N
        for b in range(B):
            want = {}
            v_ref = QD.step(cfg, W, lats[b], prompts[b], sig, h, w, state=states[b],
                            probe=lambda name, a: want.__setitem__(name, a))
            prev = got[("x_in", -1)].reshape(B, T, D)[b]
            prev_want = np.concatenate([want["txt_in"], want["img_in"]]) if step_i == 0 else want["img_in"]
            for i in range(NB):
                out = got[("block", i)].reshape(B, T, D)[b]
                _check_block(out, want[f"block{i}"], f"step {step_i} block {i}")
                _check_delta(out, prev, want[f"block{i}"], prev_want, f"step {step_i} block {i}")
                prev, prev_want = out, want[f"block{i}"]
            assert _rel(vel[b], v_ref) < MAX_REL and _cos(vel[b], v_ref) >= MIN_COS
        lats = [l * 0.9 for l in lats]


def test_config1_block_full_width(cuda):
    """one qwen1 block at hidden 3072, 24 heads, FFN 12288, 1024 image + 128 text tokens
    (text 3584 -> 3072), batch 1, sigma 0.5."""
    D, H, F, NB, TD = 3072, 24, 12288, 1, 3584
    h = w = 32
    S, B = 128, 1
    N = h * w
    d, cfg = _make(0, D, H, F, NB, TD, B, S, N, seed=1)
    W = d.weights()
    prompts, lats = _inputs(B, S, N, TD, seed=2)
    d.begin(prompts[0], h, w, slot=0)
    got = {}
    d.set_probe(lambda name, layer, a: got.__setitem__((name, layer), a))
    vel = d.step(lats[0], 0.5, slot=0)
    d.set_probe(None)
    want = {}
    v_ref = QD.step(cfg, W, lats[0], prompts[0], 0.5, h, w, probe=lambda name, a: want.__setitem__(name, a))
    out = np.concatenate([got[("block.txt", 0)].reshape(S, D), got[("block.img", 0)].reshape(N, D)])
    _check_block(out, want["block0"], "config 1 block")
    _check_delta(out, np.concatenate([got[("txt_in", -1)].reshape(S, D), got[("img_in", -1)].reshape(N, D)]),
                 want["block0"], np.concatenate([want["txt_in"], want["img_in"]]), "config 1 block")
    assert _rel(vel, v_ref) < MAX_REL and _cos(vel, v_ref) >= MIN_COS


@pytest.mark.parametrize("variant", [0, 1])
def test_strong_modulation_block_contributions(cuda, variant):
    """Weights whose modulation is of order one (the time MLP and modulation matrices scaled up, per-head norm
    weights 1 + 0.5 N(0, 1)), the regime in which the inferred choices (tanh gates, per-row modulation, norm before
    RoPE, interleaved RoPE pairs) change a block's contribution beyond tolerance (tests/test_semantics_cpu.py): every
    block's contribution and the velocity against the oracle; for ref21 a second, cached-text step too."""
    from tests.test_semantics_cpu import STRONG_MOD

    D, H, F, NB, TD = 256, 2, 512, 2, 128
    h, w, S = 6, 7, 9
    N = h * w
    d, cfg = _make(variant, D, H, F, NB, TD, 1, S, N, seed=13)
    for i, (name, shape) in enumerate(d.weight_names()):
        key = name.split(".", 1)[1] if name.startswith("blk") else name
        if name.endswith(("norm_q", "norm_k")) or name == "txt_norm.w":
            d.write_weight(name, 1.0 + 0.5 * rng.normal(rng.tensor_key(15, i), shape[0]))
        elif key in STRONG_MOD:
            d.write_weight(name, d.read_weight(name, shape) * STRONG_MOD[key])
    W = d.weights()
    prompts, lats = _inputs(1, S, N, TD, seed=16)
    d.begin(prompts[0], h, w, slot=0)
    state = {} if variant == 1 else None
    for step_i, sig in enumerate([0.6, 0.45] if variant == 1 else [0.6]):
        got = {}
        d.set_probe(lambda name, layer, a: got.__setitem__((name, layer), a))
        vel = d.step(lats[0], sig, slot=0)
        d.set_probe(None)
        want = {}
        v_ref = QD.step(cfg, W, lats[0], prompts[0], sig, h, w, state=state,
                        probe=lambda name, a: want.__setitem__(name, a))
        if variant == 0:
            prev = np.concatenate([got[("txt_in", -1)].reshape(S, D), got[("img_in", -1)].reshape(N, D)])
            outs = [np.concatenate([got[("block.txt", i)].reshape(S, D), got[("block.img", i)].reshape(N, D)])
                    for i in range(NB)]
        else:
            prev = got[("x_in", -1)].reshape(-1, D)
            outs = [got[("block", i)].reshape(-1, D) for i in range(NB)]
        prev_want = np.concatenate([want["txt_in"], want["img_in"]]) if step_i == 0 else want["img_in"]
        for i in range(NB):
            _check_delta(outs[i], prev, want[f"block{i}"], prev_want, f"step {step_i} block {i}")
            prev, prev_want = outs[i], want[f"block{i}"]
        assert _rel(vel, v_ref) < MAX_REL and _cos(vel, v_ref) >= MIN_COS, (_rel(vel, v_ref), _cos(vel, v_ref))


def test_step_cfg_matches_two_steps(cuda):
    """mkb_dit_step_cfg (cond + uncond batched, CFG and Euler fused on the device) against two single steps
    combined on the host as Engine::generate does (engine.cpp:475-480, 500-503)."""
    D, H, F, NB, TD = 512, 4, 1024, 2, 256
    h, w, S = 8, 8, 16
    N = h * w
    d, _ = _make(0, D, H, F, NB, TD, 2, S, N, seed=9)
    prompts, lats = _inputs(2, S, N, TD, seed=4)
    d.begin(prompts[0], h, w, slot=0)
    d.begin(prompts[1], h, w, slot=1)
    x = lats[0]
    vc = d.step(x, 0.7, slot=0)
    vu = d.step(x, 0.7, slot=1)
    want = x + (0.55 - 0.7) * (vu + 4.0 * (vc - vu))
    got = d.step_cfg(x, 0.7, 0.55, 4.0)
    assert np.abs(got - want).max() < 1e-4


def test_graph_replay_matches_eager(cuda):
    """The step body runs eagerly on a geometry's first call, is captured as a CUDA graph on the second and replayed
    after. Alternating latents make a replay that did no work visible (it would return the previous call's result).
    qwen1 also with one block: its modulation then has no side-stream part, which the capture must not fork."""
    for variant, blocks in ((0, 2), (0, 1), (1, 2)):
        d, cfg = _make(variant, 512, 4, 1024, blocks, 256, 2, 20, 64, seed=21)
        prompts, lats = _inputs(2, 20, 64, 256, seed=8)
        a = np.stack(lats)
        b = a[::-1].copy() * 0.5
        c = a * 0.25
        d.begin(prompts[0], 8, 8, slot=0)
        d.begin(prompts[1], 8, 8, slot=1)
        if variant == 0:  # eager, capture, replay, replay
            o = [d.step_batch([0, 1], x, [0.4, 0.4]) for x in (a, b, a, b)]
            assert not np.allclose(o[0], o[1])
            assert np.array_equal(o[2], o[0]) and np.array_equal(o[3], o[1])
        else:  # the first step (text rows) is its own geometry; then eager, capture, replay of the cached-text step
            d.step_batch([0, 1], a, [0.9, 0.9])
            o = [d.step_batch([0, 1], x, [0.4, 0.4]) for x in (b, c, b, c)]
            assert not np.allclose(o[0], o[1])
            assert np.array_equal(o[2], o[0]) and np.array_equal(o[3], o[1])
