"""Small DiT step, UNet step and VAE decode with fixed seeds, shared by tests/test_launch_overlap_gpu.py and its child
process. Run as a script (`python tests/launch_cases.py out.npz`) it saves the outputs, so a process started with
MKB_PDL=0 (kernels launched without programmatic dependent launch) can be compared bit for bit."""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run():
    import numpy as np
    import mkimage
    from oracle import rng

    out = {}
    # DiT (qwen1 blocks), two steps through the host API; the second replays the captured graph.
    D, H, F, NB, TD, h, w, S = 512, 4, 1024, 2, 256, 8, 8, 16
    d = mkimage.Dit(mkimage.DitConfig(variant=mkimage.QWEN1, hidden=D, heads=H, ffn=F, blocks=NB, text_dim=TD,
                                      max_batch=2, max_text_tokens=S, max_image_tokens=h * w, slots=2))
    d.init_random(3)
    prompt = rng.normal(rng.tensor_key(5, 0), S * TD).reshape(S, TD)
    lat = rng.normal(rng.tensor_key(5, 1), h * w * 64).reshape(h * w, 64)
    d.begin(prompt, h, w, slot=0)
    out["dit_step1"] = d.step(lat, 0.5, slot=0)
    out["dit_step2"] = d.step(lat, 0.5, slot=0)
    d.close()
    # UNet, three batched steps (eager, captured, replayed).
    cfg = dict(channels=(64, 128, 256), depth=(0, 1, 2), layers=2, context_dim=256, pooled_dim=128)
    gh, gw, S, B = 16, 16, 77, 2
    u = mkimage.Unet(mkimage.UnetConfig(max_batch=B, max_gh=gh, max_gw=gw, max_context=S, slots=2, **cfg))
    u.init_random(17)
    for b in range(B):
        ctx = rng.normal(rng.tensor_key(3, 10 + b), S * 256).reshape(S, 256)
        u.begin(ctx, rng.normal(rng.tensor_key(3, 20 + b), 128), gh, gw, slot=b)
    lats = np.stack([rng.normal(rng.tensor_key(3, 30 + b), gh * gw * 16).reshape(gh * gw, 16) * 3.0
                     for b in range(B)])
    for i in range(3):
        out[f"unet_step{i}"] = u.step_batch(lats, [2.5, 7.0])
    # VAE decode.
    v = mkimage.Vae(mkimage.VaeConfig(max_gh=8, max_gw=8, channels=(128, 128, 256, 256), layers=1))
    v.init_random(23)
    out["vae"] = v.decode(rng.normal(rng.tensor_key(4, 1), 64 * 16).reshape(64, 16) * 0.13025, 8, 8)
    return {k: np.asarray(a, np.float32) for k, a in out.items()}, mkimage.ops.check_kernels()


if __name__ == "__main__":
    for p in (ROOT, os.path.join(ROOT, "mako-image_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import numpy as np

    res, st = run()
    np.savez(sys.argv[1], status=np.array(st), **res)
