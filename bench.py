"""Benchmark of the B200 denoiser hot path: Qwen-Image-shape MMDiT denoising steps per second.

Default: the full 60-block Qwen-Image-shape MMDiT (hidden 3072, 24 heads x 128, FFN 12288
GELU, text 3584 -> 3072) at 1024^2 (4096 image + 256 text tokens), CFG batch 2 (cond / uncond in one pass), the
Euler update fused on the device. One "step" = one guided denoising step of one image. Weights are random bf16
N(0, 0.02) generated on the device by seed; prompt and latents are seeded synthetic normals.

  python bench.py [--gpus N --steps K --warmup W] [--impl mkb|reference] [--config 1|2|5]

Under torchrun (N > 1) every rank runs its own image on its own GPU (weak scaling: CFG pairs are independent, no
collective on the data path); value = images*steps over the max-over-ranks device time.

--impl reference times the reference's math on the host CPU cores instead: the oracle port (oracle/qwen_dit.py,
numpy/BLAS) on a bounded sample (one block of one sample, scaled to the full step), since the reference's own
implementation (Metal) cannot run here.
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "mako-image_b200"))
sys.path.insert(0, ROOT)

METRIC = "Qwen-Image-shape DiT steps/s at 1024^2 (CFG batch 2, Euler fused)"
UNIT = "steps/s"

CONFIGS = {
    # name: (grid h, grid w, text tokens, images, blocks)
    3: dict(workload="SDXL UNet step, 1024^2, CFG batch 2 (BASELINE configs[2])"),
    4: dict(workload="SDXL VAE decode, 1024^2 (BASELINE configs[3])"),
    1: dict(h=32, w=32, S=128, images=1, blocks=1, cfg=False,
            workload="qwen1 MMDiT, 1 block, 1024 image + 128 text tokens, batch 1 (BASELINE configs[0])"),
    2: dict(h=64, w=64, S=256, images=1, blocks=60, cfg=True,
            workload="qwen1 MMDiT, 60 blocks, 1024^2 (4096 image + 256 text tokens), CFG batch 2, Euler fused "
                     "(BASELINE configs[1])"),
    5: dict(h=128, w=128, S=1024, images=4, blocks=60, cfg=True,
            workload="qwen1 MMDiT, 60 blocks, 2048^2 (16384 image + 1024 text tokens), CFG batch 2 x 4 images "
                     "(BASELINE configs[4]) on one GPU per rank"),
}
D, H, F, TD = 3072, 24, 12288, 3584


def _peaks():
    """(burst bf16 TFLOP/s, HBM GB/s, kind). The burst figure is the denominator for a kernel timed alone."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p["bf16_tflops"], p["hbm_gbs"], "measured"
    except Exception:
        return 1590.0, 6650.0, "fallback"


def _sustained_peak():
    """(bf16 TFLOP/s, kind) for work timed inside a long step: cuBLAS back to back for seconds under the power cap."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)["bf16_tflops_sustained"], "measured sustained"
    except Exception:
        return 1400.0, "fallback sustained"


def _step_fracs(step_tflops):
    """Step throughput as fractions of the sustained peak (the denominator for a long step) and of the burst one."""
    burst, _, burst_kind = _peaks()
    sus, sus_kind = _sustained_peak()
    return {"step_tflops": step_tflops, "step_peak": sus, "step_peak_kind": sus_kind,
            "step_frac": step_tflops / sus, "step_frac_of_burst": step_tflops / burst}


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


_CPU_CACHE = {}


def cpu_baseline(cfg, reps=1):
    """The oracle port (numpy; BLAS threads on the host cores) on a bounded sample: one qwen1 block of one sample at
    the config's shape. Returns seconds per full step (scaled by blocks x samples) and the sample description."""
    import numpy as np
    from oracle import qwen_dit as QD

    try:
        from threadpoolctl import threadpool_info

        cores = max([i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"] or [1])
    except Exception:
        cores = os.cpu_count() or 1
    h, w, S = cfg["h"], cfg["w"], cfg["S"]
    N = h * w
    oc = QD.default_cfg("qwen1", D, H, F, 1, TD)
    r = np.random.default_rng(0)
    if "W" not in _CPU_CACHE:
        W = {}
        for name, shape in QD.weight_shapes(oc).items():
            if name.endswith(("norm_q", "norm_k", "txt_norm.w")):
                W[name] = np.ones(shape, np.float32)
            else:
                W[name] = (r.standard_normal(shape, dtype=np.float32) * 0.02)
        _CPU_CACHE["W"] = W
    W = _CPU_CACHE["W"]
    prompt = r.standard_normal((S, TD), dtype=np.float32)
    lat = r.standard_normal((N, 64), dtype=np.float32)
    # time the block alone (the step's inputs prepared outside the timed region)
    st = np.ones(D, np.float32) * 0.1
    rope = QD.rope_table(oc, S, h, w)
    x_txt = QD.text_in(oc, W, prompt)
    x_img = lat @ W["img_in.w"].T
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        QD.block_qwen1(oc, W, 0, x_txt, x_img, st, rope)
        times.append(time.perf_counter() - t0)
    t_block = min(times)
    samples = cfg["images"] * (2 if cfg["cfg"] else 1)
    t_step = t_block * cfg["blocks"] * samples
    sample = (f"one qwen1 block of one sample ({N} image + {S} text tokens), {t_block:.2f} s, scaled x "
              f"{cfg['blocks']} blocks x {samples} samples (extrapolated from 1 block)")
    return t_step, cores, sample


def run_reference(args, cfg):
    ws, rank, _ = _dist()
    if rank != 0:
        return
    for _ in range(args.warmup):
        cpu_baseline(cfg)
    secs = []
    for _ in range(args.steps):
        t, cores, sample = cpu_baseline(cfg)
        secs.append(t)
    t_step = statistics.mean(secs)
    v = 1.0 / t_step
    samples = cfg["images"] * (2 if cfg["cfg"] else 1)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_step * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "extrapolated_from": "1 block of 1 sample per step (x %d blocks x %d samples): steps x ms_per_step is "
                                 "not the time this run measured" % (cfg["blocks"], samples),
            "measured_ms_per_block": t_step * 1e3 / (cfg["blocks"] * samples),
            "config": {"workload": cfg["workload"], "impl_detail": "oracle port (numpy + BLAS) on host cores"},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def cfg_pair_group(dist, ws, rank):
    """The process group of this rank's CFG pair when cond and uncond of one image sit on ranks 2i and 2i + 1.
    new_group is collective, so every rank creates every pair's group and keeps its own."""
    mine = None
    for r0 in range(0, ws, 2):
        grp = dist.new_group([r0, r0 + 1])
        if rank // 2 == r0 // 2:
            mine = grp
    return mine


def run_mkb(args, cfg):
    import numpy as np
    import torch
    import mkimage
    from oracle import rng

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=dev)
    h, w, S, n_img = cfg["h"], cfg["w"], cfg["S"], cfg["images"]
    N = h * w
    split_mode = args.split_samples and ws > 1
    half_pair = False  # sample split with one sample (half a CFG pair) per rank
    if split_mode:
        # The job's images spread over the ranks, whole CFG pairs per rank while there are enough (strong scaling:
        # the total work is fixed); with twice as many ranks as images, cond and uncond of one image sit on two
        # neighbouring ranks, which exchange their predictions for the guided update.
        if not cfg["cfg"] or (n_img % ws and ws != 2 * n_img):
            raise SystemExit(f"--split-samples: {n_img} CFG pairs do not divide over {ws} ranks")
        half_pair = ws == 2 * n_img
        n_img = 1 if half_pair else n_img // ws
    B = 1 if half_pair else n_img * (2 if cfg["cfg"] else 1)
    d = mkimage.Dit(mkimage.DitConfig(variant=mkimage.QWEN1, hidden=D, heads=H, ffn=F, blocks=cfg["blocks"],
                                      text_dim=TD, max_batch=B, max_text_tokens=S, max_image_tokens=N, slots=B))
    d.init_random(seed=1234)
    sp_mode = args.sp and ws > 1
    if sp_mode:
        # One sequence-parallel group over all ranks: rank 0's NCCL id to every rank, then the collective set-up.
        obj = [mkimage.nccl_unique_id() if rank == 0 else None]
        torch.distributed.broadcast_object_list(obj, src=0)
        d.set_sequence_parallel(obj[0], rank, ws)
        if args.sp_exchange.startswith("heads") and H % ws:
            args.sp_exchange = "peer"  # the head split needs the heads to divide over the ranks
        if args.sp_exchange == "peer":
            d.set_peer_exchange(True)
        elif args.sp_exchange == "heads":
            d.set_head_exchange(1)
        elif args.sp_exchange == "heads_peer":
            d.set_head_exchange(2)
    for s in range(B):
        prompt = rng.normal(rng.tensor_key(99, (rank % 2) if half_pair else s), S * TD).reshape(S, TD)
        d.begin(prompt, h, w, slot=s)
    # Replicas step their own images; a sequence-parallel group steps the same images on every rank; split samples
    # step their share of the job's images (both ranks of a split pair the same latents).
    lat_key = 0 if sp_mode else (rank // 2 if half_pair else rank)
    lat_host = rng.normal(rng.tensor_key(98, lat_key), n_img * N * 64).reshape(n_img, N, 64)
    lat = torch.from_numpy(lat_host).to(dev)
    sig = mkimage.sigmas(40, N)
    i0 = int(np.argmin(np.abs(sig[:-1] - 0.5)))
    sigma, sigma_next = float(sig[i0]), float(sig[i0 + 1])
    # One explicit stream for the library's launches and the CUDA events that time them.
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    sp = mkimage.stream_ptr(stream)

    pair_group = None
    if half_pair:
        pair_group = cfg_pair_group(torch.distributed, ws, rank)
        vel = torch.empty(N * 64, device=dev)
        both = torch.empty(2, N * 64, device=dev)
        guided = torch.empty(N * 64, device=dev)

    def one_step():
        if half_pair:
            # This rank's prediction, the partner's by an all-gather of the pair, then the same guided Euler update
            # on both ranks (rank 2i holds the prompt, 2i + 1 the negative).
            d.step_batch_dev([0], lat.data_ptr(), [sigma], vel.data_ptr(), sp)
            torch.distributed.all_gather_into_tensor(both, vel, group=pair_group)
            mkimage.check(mkimage.lib.mkb_cfg_combine_dev(guided.data_ptr(), both[0].data_ptr(), both[1].data_ptr(),
                                                          4.0, N * 64, sp))
            mkimage.check(mkimage.lib.mkb_axpy_dev(lat.data_ptr(), guided.data_ptr(), sigma_next - sigma, N * 64, sp))
        elif cfg["cfg"]:
            d.step_cfg_dev(n_img, lat.data_ptr(), sigma, sigma_next, 4.0, sp)
        else:
            out = torch.empty_like(lat)
            d.step_batch_dev([0], lat.data_ptr(), [sigma], out.data_ptr(), sp)

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    launches0 = mkimage.lib.mkb_kernel_launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.nvtx.range_push("mkb_timed")
        e0.record(stream)
        for _ in range(args.steps):
            one_step()
        e1.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    launches = mkimage.lib.mkb_kernel_launches() - launches0
    ms = e0.elapsed_time(e1) / args.steps
    mkimage.ops.check_kernels()
    if ws > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = t.item()
        torch.distributed.barrier()
    job_images = cfg["images"] if (sp_mode or split_mode) else n_img * ws
    value = job_images * 1e3 / ms
    flops_step = d.step_flops(B) / (ws if sp_mode else 1)  # this rank's share of the step

    # End to end through the public host-buffer API: pinned latents in, updated latents out, every step.
    e2e = None
    if cfg["cfg"] and n_img == 1 and not half_pair:
        pinned = torch.from_numpy(lat_host[0].copy()).pin_memory()
        guided = d.step_cfg_inplace(pinned.numpy())  # H2D from and D2H into the pinned buffer every step
        for _ in range(2):
            guided(sigma, sigma_next, 4.0)
        if ws > 1:
            torch.distributed.barrier()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            guided(sigma, sigma_next, 4.0)
        t_e2e = (time.perf_counter() - t0) / args.steps
        if ws > 1:
            t = torch.tensor([t_e2e], device=dev)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            t_e2e = t.item()
        e2e = {"value": job_images / t_e2e, "unit": UNIT, "h2d_bytes_per_step": N * 64 * 4,
               "d2h_bytes_per_step": N * 64 * 4}

    # Roofline: each of the block's hot kernels timed alone on the same stream with CUDA events at the step's
    # shapes; the dominant one (the FFN-up GEMM) is the line's `kernel`, the table gives all five and the
    # time-weighted fraction of one block's set.
    peak_tf, peak_hbm, peak_kind = _peaks()
    table = {}
    for name, (fn, work) in hot_kernels(dev, cfg).items():
        kms = time_kernel(fn, stream)
        table[name] = {"ms": kms, "achieved": work / (kms * 1e-3) / 1e12, "frac": work / (kms * 1e-3) / 1e12 / peak_tf,
                       "gflop": work / 1e9}
    mkimage.ops.check_kernels()
    achieved = table["ffn_up"]["achieved"]
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "gemm_ffn_up_config2.md")) as f:
            for ln in f:
                if ln.startswith("dram_bytes_per_launch:"):
                    traffic = float(ln.split(":")[1])
    except Exception:
        pass
    block_work = sum(t["gflop"] for t in table.values()) * 1e9
    block_ms = sum(t["ms"] for t in table.values())
    roofline = {"bound": "tensor", "kernel": "k_gemm2 (tcgen05 CTA pair, 256x256 tiles, FFN-up 8192x12288x3072, "
                                              "GELU epilogue)",
                "achieved": achieved, "peak": peak_tf, "peak_kind": peak_kind, "unit": "TFLOP/s",
                "frac": achieved / peak_tf, "traffic": traffic,
                "kernels": table,
                "block_time_weighted_frac": block_work / (block_ms * 1e-3) / 1e12 / peak_tf,
                **_step_fracs(flops_step / (ms * 1e-3) / 1e12)}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        t_step, cores, sample = cpu_baseline(cfg)
        cpu = {"value": n_img / t_step, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample}

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
                "scaling": "strong" if (sp_mode or split_mode) else "weak",
                "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": cfg["workload"], "hidden": D, "heads": H, "ffn": F, "blocks": cfg["blocks"],
                           "image_tokens": N, "text_tokens": S, "samples_per_gpu": B,
                           "parallelism": (f"sequence parallel x{ws} (each rank 1/{ws} of every sample's joint rows, "
                                           + ("K/V shards pushed into the peers' memory by copy engines during the "
                                              "attention)" if args.sp_exchange == "peer" else
                                              f"q/k/v all-to-all to {H // ws} heads per rank and outputs back, per "
                                              "block over NCCL)" if args.sp_exchange == "heads" else
                                              f"q/k/v of {H // ws} heads per rank and the outputs stored into the "
                                              "peers' memory by the QKV and attention epilogues)"
                                              if args.sp_exchange == "heads_peer" else
                                              "K/V all-gathered per block over NCCL)")) if sp_mode else
                                          (f"sample split x{ws} ({cfg['images']} images, "
                                           + ("cond / uncond of an image on neighbouring ranks, predictions "
                                              "all-gathered per step)" if half_pair else
                                              f"{n_img} whole CFG pairs per rank, no collective)"))
                                          if split_mode else
                                          f"replicas x{ws} (images per GPU as configured, CFG pair batched)",
                           "l2": "inputs larger than L2 (40.8 GB of weights streamed per step)",
                           "step_tflop": flops_step / 1e12},
                "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "clocks": clk.summary(),
                "gpu_launches": int(launches)}
        print(json.dumps(line), flush=True)
    d.close()
    if ws > 1:
        torch.distributed.destroy_process_group()


SDXL_UNET = dict(channels=(320, 640, 1280), depth=(0, 2, 10), layers=2, context_dim=2048, pooled_dim=1280)
SDXL_VAE = dict(channels=(128, 256, 512, 512), layers=2)


def unet_flops(oc, gh, gw, S, B):
    """Algorithmic FLOPs of one UNet pass (convolutions, transformer linears, attention) from the block list."""
    from oracle import sdxl as OS

    f, h, w, c = 0.0, 2 * gh, 2 * gw, 4
    for op in OS.unet_structure(oc):
        P = h * w
        if op[0] == "conv_in":
            f += 2 * P * op[2] * 9 * 4
        elif op[0] == "res":
            _, _, cin, cout = op
            f += 2 * P * cout * 9 * (cin + cout) + (2 * P * cout * cin if cin != cout else 0)
        elif op[0] == "attn":
            cc, d = op[2], op[3]
            f += 4 * P * cc * cc + d * (36 * P * cc * cc + 4 * P * P * cc + 4 * P * S * cc)
        elif op[0] == "down":
            h, w = h // 2, w // 2
            f += 2 * h * w * op[2] * 9 * op[2]
        elif op[0] == "up":
            h, w = h * 2, w * 2
            f += 2 * h * w * op[2] * 9 * op[2]
    return (f + 2 * 4 * gh * gw * 4 * 9 * oc["channels"][0]) * B


def vae_flops(vc, gh, gw):
    from oracle import sdxl as OS

    h, w = 2 * gh, 2 * gw
    f = 2 * h * w * vc["channels"][-1] * 9 * 4
    for op in OS.vae_structure(vc)[2:]:
        P = h * w
        if op[0] == "res":
            _, _, cin, cout = op
            f += 2 * P * cout * 9 * (cin + cout) + (2 * P * cout * cin if cin != cout else 0)
        elif op[0] == "attn":
            f += 8 * P * op[2] * op[2] + 4 * P * P * op[2]
        elif op[0] == "up":
            h, w = h * 2, w * 2
            f += 2 * h * w * op[2] * 9 * op[2]
    return f + 2 * h * w * 3 * 9 * vc["channels"][0]


def sdxl_cpu_baseline(kind):
    """The oracle port on the host cores at 256^2 (full widths; UNet transformer depths 1/1 to bound the run),
    scaled to the 1024^2 workload by the FLOP ratio. Returns (seconds per full unit, cores, sample)."""
    import numpy as np
    from oracle import sdxl as OS

    try:
        from threadpoolctl import threadpool_info

        cores = max([i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"] or [1])
    except Exception:
        cores = os.cpu_count() or 1
    r = np.random.default_rng(0)

    def weights(shapes):
        W = {}
        for k, shp in shapes.items():
            norm = k.endswith((".gn.w", ".gn1.w", ".gn2.w", ".ln1.w", ".ln2.w", ".ln3.w", "out.gn.w"))
            W[k] = np.ones(shp, np.float32) if norm else r.standard_normal(shp, dtype=np.float32) * 0.02
        return W

    gh = gw = 16
    if kind == "unet":
        oc = OS.unet_default_cfg(depth=(0, 1, 1))
        if "unet" not in _CPU_CACHE:  # generated once per process, outside every timed call
            _CPU_CACHE["unet"] = weights(OS.unet_weight_shapes(oc))
        W = _CPU_CACHE["unet"]
        st = OS.unet_begin(oc, W, r.standard_normal((77, 2048), dtype=np.float32),
                           r.standard_normal(1280, dtype=np.float32), gh, gw)
        lat = r.standard_normal((gh * gw, 16), dtype=np.float32)
        t0 = time.perf_counter()
        OS.unet_step(oc, W, st, lat, 5.0)
        t = time.perf_counter() - t0
        full = unet_flops(OS.unet_default_cfg(**SDXL_UNET), 64, 64, 77, 2)
        small = unet_flops(oc, gh, gw, 77, 1)
        return t * full / small, cores, (f"UNet pass at 256^2, full widths, transformer depths 0/1/1 ({t:.2f} s), "
                                         f"scaled by FLOPs to 1024^2 CFG 2 (x{full / small:.1f})")
    vc = OS.vae_default_cfg(**SDXL_VAE)
    if "vae" not in _CPU_CACHE:
        _CPU_CACHE["vae"] = weights(OS.vae_weight_shapes(vc))
    W = _CPU_CACHE["vae"]
    lat = r.standard_normal((gh * gw, 16), dtype=np.float32) * 0.13
    t0 = time.perf_counter()
    OS.vae_decode(vc, W, lat, gh, gw)
    t = time.perf_counter() - t0
    full, small = vae_flops(vc, 64, 64), vae_flops(vc, gh, gw)
    return t * full / small, cores, f"VAE decode at 256^2 ({t:.2f} s), scaled by FLOPs to 1024^2 (x{full / small:.1f})"


def run_sdxl(args, which):
    """config 3 (SDXL UNet step, 1024^2, CFG batch 2, Euler fused) or 4 (SDXL VAE decode 1024^2)."""
    import numpy as np
    import torch
    import mkimage
    from oracle import rng

    ws, rank, local = _dist()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import datetime

        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    sp = mkimage.stream_ptr(stream)
    gh = gw = 64
    peak_tf, _, peak_kind = _peaks()
    if which == 3:
        metric, unit = "SDXL UNet steps/s at 1024^2 (CFG batch 2, Euler fused)", "steps/s"
        u = mkimage.Unet(mkimage.UnetConfig(max_batch=2, max_gh=gh, max_gw=gw, max_context=77, slots=2, **SDXL_UNET))
        u.init_random(seed=77)
        for s in range(2):
            u.begin(rng.normal(rng.tensor_key(50, s), 77 * 2048).reshape(77, 2048),
                    rng.normal(rng.tensor_key(51, s), 1280), gh, gw, slot=s)
        lat_host = rng.normal(rng.tensor_key(52, rank), gh * gw * 16).reshape(gh * gw, 16) * 14.6
        lat = torch.from_numpy(lat_host).to(dev)
        sig = mkimage.sdxl_sigmas(28)
        sigma, sigma_next = float(sig[10]), float(sig[11])
        one = lambda: u.step_cfg_dev(lat.data_ptr(), sigma, sigma_next, 5.0, sp)  # noqa: E731
        flops = u.step_flops(2)
        workload = "SDXL UNet (320/640/1280, depths 0/2/10, hd 64, 77x2048 context), 1024^2, CFG batch 2, Euler fused"
    else:
        metric, unit = "SDXL VAE decodes/s at 1024^2", "decodes/s"
        u = mkimage.Vae(mkimage.VaeConfig(max_gh=gh, max_gw=gw, **SDXL_VAE))
        u.init_random(seed=78)
        lat_host = rng.normal(rng.tensor_key(53, rank), gh * gw * 16).reshape(gh * gw, 16) * 0.13
        lat = torch.from_numpy(lat_host).to(dev)
        out = torch.empty(16 * gh, 16 * gw, 4, device=dev)
        one = lambda: u.decode_dev(lat.data_ptr(), gh, gw, out.data_ptr(), sp)  # noqa: E731
        flops = u.decode_flops(gh, gw)
        workload = "SDXL VAE decoder (AutoencoderKL 128/256/512/512), 128^2x4 latent -> 1024^2 RGB"
    for _ in range(args.warmup):
        one()
    torch.cuda.synchronize()
    if ws > 1:
        torch.distributed.barrier()
    launches0 = mkimage.lib.mkb_kernel_launches()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.nvtx.range_push("mkb_timed")
        e0.record(stream)
        for _ in range(args.steps):
            one()
        e1.record(stream)
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    launches = mkimage.lib.mkb_kernel_launches() - launches0
    ms = e0.elapsed_time(e1) / args.steps
    mkimage.ops.check_kernels()
    if ws > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = t.item()
    value = ws * 1e3 / ms
    # End to end through the host-buffer API (latents in, result out, every call).
    if which == 3:
        x2 = np.stack([lat_host, lat_host]).astype(np.float32)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            eps = u.step_batch(x2, [sigma, sigma])
            mkimage.guided_euler(x2[0], eps[0], eps[1], 5.0, sigma, sigma_next)
        t_e2e = (time.perf_counter() - t0) / args.steps
        e2e = {"value": 1.0 / t_e2e, "unit": unit, "h2d_bytes_per_step": x2.nbytes, "d2h_bytes_per_step": x2.nbytes}
    else:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            img = u.decode(lat_host, gh, gw)
        t_e2e = (time.perf_counter() - t0) / args.steps
        e2e = {"value": 1.0 / t_e2e, "unit": unit, "h2d_bytes_per_step": lat_host.astype(np.float32).nbytes,
               "d2h_bytes_per_step": img.nbytes}
    # Dominant kernel: the implicit-GEMM 3x3 convolution (level-2 UNet 1280 -> 1280 at 32^2 x 2 samples; VAE
    # 256 -> 256 at 512^2), timed alone on the same stream.
    if which == 3:
        B_, H_, W_, C_ = 2, 32, 32, 1280
    else:
        B_, H_, W_, C_ = 1, 512, 512, 256
    xa = torch.randn(B_, H_, W_, C_, device=dev).to(torch.bfloat16)
    wa = (torch.randn(C_, 9 * C_, device=dev) * 0.02).to(torch.bfloat16)
    ya = torch.empty(B_, H_, W_, C_, device=dev)
    for _ in range(3):
        mkimage.ops.conv2d(xa, wa, out=ya)
    g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g0.record(stream)
    for _ in range(10):
        mkimage.ops.conv2d(xa, wa, out=ya)
    g1.record(stream)
    torch.cuda.synchronize()
    cms = g0.elapsed_time(g1) / 10
    cfl = 2.0 * B_ * H_ * W_ * C_ * 9 * C_
    ach = cfl / (cms * 1e-3) / 1e12
    roofline = {"bound": "tensor", "kernel": f"k_gemm conv mode (3x3, {C_}->{C_} at {H_}x{W_} x{B_})",
                "achieved": ach, "peak": peak_tf, "peak_kind": peak_kind, "unit": "TFLOP/s", "frac": ach / peak_tf,
                "traffic": None, **_step_fracs(flops / (ms * 1e-3) / 1e12)}
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        t_unit, cores, sample = sdxl_cpu_baseline("unet" if which == 3 else "vae")
        cpu = {"value": 1.0 / t_unit, "unit": unit, "cores": cores, "kind": "port", "sample": sample}
    if rank == 0:
        print(json.dumps({"metric": metric, "value": value, "unit": unit, "n_gpus": ws, "steps": args.steps,
                          "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
                          "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                          "config": {"workload": workload, "tflop_per_step": flops / 1e12,
                                     "parallelism": f"replicas x{ws}", "l2": "activations and weights above L2"},
                          "e2e": e2e, "roofline": roofline, "cpu_baseline": cpu, "clocks": clk.summary(),
                          "gpu_launches": int(launches)}), flush=True)
    u.close()
    if ws > 1:
        torch.distributed.destroy_process_group()


def hot_kernels(dev, cfg, names=None):
    """The block's hot kernels at the config's image-row shapes (CFG batch rows together), each as (launch, FLOPs):
    qkv (the fused QKV projection with per-head RMSNorm + RoPE into the attention layout), attention (joint, all
    L = S + N keys), oproj (the O-projection with the gated residual reduce-added by TMA), ffn_up (GELU epilogue),
    ffn_down (gated residual). Synthetic inputs of the right shapes; weights N(0, 0.02)."""
    import torch
    import mkimage

    h, w, S, n_img = cfg["h"], cfg["w"], cfg["S"], cfg["images"]
    N = h * w
    B = n_img * (2 if cfg["cfg"] else 1)
    L = S + N
    M = B * N
    g = torch.Generator(device=dev).manual_seed(0)
    out = {}
    names = names or ["qkv", "attention", "oproj", "ffn_up", "ffn_down"]

    def mat(r, c, sd=1.0):
        return (torch.randn(r, c, device=dev, generator=g) * sd).to(torch.bfloat16)

    if "qkv" in names:
        x, wq = mat(M, D), mat(3 * D, D, 0.02)
        bq = torch.zeros(3 * D, device=dev)
        nq, nk = torch.ones(128, device=dev), torch.ones(128, device=dev)
        rope = torch.zeros(L, 64, 2, device=dev)
        rope[..., 0] = 1.0
        qh = torch.empty(B, H, L, 128, device=dev, dtype=torch.bfloat16)
        kh, vh = torch.empty_like(qh), torch.empty_like(qh)
        out["qkv"] = (lambda: mkimage.ops.proj_qkv_heads(x, wq, bq, nq, nk, rope, qh, kh, vh, N, S),
                      2.0 * M * 3 * D * D)
    if "attention" in names:
        q = torch.randn(B, H, L, 128, device=dev, generator=g).to(torch.bfloat16)
        k, v = torch.randn_like(q), torch.randn_like(q)
        o0 = torch.empty(B * S, D, device=dev, dtype=torch.bfloat16)
        o1 = torch.empty(B * N, D, device=dev, dtype=torch.bfloat16)
        out["attention"] = (lambda: mkimage.ops.attention(q, k, v, o0, o1, split=S), 4.0 * B * L * L * D)
    if "oproj" in names or "ffn_down" in names:
        resid = torch.randn(M, D, device=dev, generator=g)
        gate = torch.randn(B, D, device=dev, generator=g) * 0.1
        bd = torch.zeros(D, device=dev)
        if "oproj" in names:
            xo, wo = mat(M, D), mat(D, D, 0.02)
            out["oproj"] = (lambda: mkimage.ops.proj_gate_add(xo, wo, resid, gate, bias=bd, rows_per_sample=N),
                            2.0 * M * D * D)
        if "ffn_down" in names:
            xf, wf = mat(M, F), mat(D, F, 0.02)
            out["ffn_down"] = (lambda: mkimage.ops.proj_gate_add(xf, wf, resid, gate, bias=bd, rows_per_sample=N),
                               2.0 * M * D * F)
    if "ffn_up" in names:
        xu, wu = mat(M, D), mat(F, D, 0.02)
        bu = torch.zeros(F, device=dev)
        yu = torch.empty(M, F, device=dev, dtype=torch.bfloat16)
        out["ffn_up"] = (lambda: mkimage.ops.proj(xu, wu, bu, act=mkimage.ops.ACT_GELU_TANH, out=yu),
                         2.0 * M * F * D)
    return out


def vae_kernel(dev, name):
    """The VAE decoder's hot kernels at config 4's shapes (1024^2 output, 128^2 latent), as (launch, FLOPs):
    vae_attention, the mid block's single-head attention over the 128^2 latent pixels at 512 channels (q | k | v rows
    side by side, as the VAE's QKV projection writes them); vae_conv128, a 3x3 convolution 128 -> 128 at 1024^2 with
    bias and residual (the last level's conv2)."""
    import torch
    import mkimage

    g = torch.Generator(device=dev).manual_seed(0)
    if name == "vae_attention":
        n, d = 128 * 128, 512
        qkv = torch.randn(n, 3 * d, device=dev, generator=g).to(torch.bfloat16)
        out = torch.empty(n, d, device=dev, dtype=torch.bfloat16)
        return (lambda: mkimage.ops.attention_wide(qkv, d, out=out)), 4.0 * n * n * d
    hw, c = 1024, 128
    x = torch.randn(1, hw, hw, c, device=dev, generator=g).to(torch.bfloat16)
    w = (torch.randn(c, 9 * c, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    b = torch.zeros(c, device=dev)
    res = torch.randn(1, hw, hw, c, device=dev, generator=g)
    out = torch.empty(1, hw, hw, c, device=dev)
    return (lambda: mkimage.ops.conv2d(x, w, bias=b, resid=res, out=out)), 2.0 * hw * hw * c * 9 * c


def time_kernel(fn, stream, reps=20, warmup=3):
    """Mean milliseconds per launch over `reps` back-to-back launches, CUDA events on the launching stream."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def run_kernel(args, cfg):
    """One hot kernel alone at the config's shape, for profiling (see hot_kernels): 3 warm-up launches then 3 timed
    ones (CUDA events)."""
    import torch
    import mkimage

    dev = torch.device("cuda", 0)
    name = {"gemm": "ffn_up"}.get(args.kernel, args.kernel)
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)
    if name.startswith("vae_"):
        fn, work = vae_kernel(dev, name)
    else:
        fn, work = hot_kernels(dev, cfg, [name])[name]
    ms = time_kernel(fn, stream, reps=3)
    mkimage.ops.check_kernels()
    print(json.dumps({"kernel": name, "config": cfg["workload"], "ms": ms, "achieved": work / (ms * 1e-3) / 1e12,
                      "unit": "TFLOP/s"}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["mkb", "reference"], default="mkb")
    ap.add_argument("--config", type=int, choices=sorted(CONFIGS), default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--split-samples", action="store_true",
                    help="DiT configs under torchrun: the config's images spread over the ranks (strong scaling)")
    ap.add_argument("--sp", action="store_true",
                    help="DiT configs under torchrun: one sequence-parallel group over all ranks instead of replicas")
    ap.add_argument("--sp-exchange", choices=["peer", "nccl", "heads", "heads_peer"], default="heads_peer",
                    help="--sp: K/V shards pushed into the peers' memory by copy engines during the attention "
                         "(peer), all-gathered by NCCL before it (nccl), or q/k/v exchanged all-to-all so that "
                         "each rank attends over whole sequences of heads / ranks heads (heads), the same with the "
                         "QKV and attention epilogues storing into the peers' memory (heads_peer, the default; "
                         "peer when the heads do not divide over the ranks)")
    ap.add_argument("--kernel", choices=["gemm", "qkv", "attention", "oproj", "ffn_up", "ffn_down", "vae_attention",
                                         "vae_conv128"], default=None,
                    help="run one hot kernel alone at the config's shape (profiling)")
    args = ap.parse_args()
    cfg = CONFIGS[args.config]
    if args.kernel:
        run_kernel(args, cfg)
    elif args.config in (3, 4) and args.impl != "reference":
        run_sdxl(args, args.config)
    elif args.config in (3, 4):
        ws, rank, _ = _dist()
        if rank == 0:
            kind = "unet" if args.config == 3 else "vae"
            for _ in range(args.warmup):
                sdxl_cpu_baseline(kind)
            secs = [sdxl_cpu_baseline(kind) for _ in range(args.steps)]
            t_unit = statistics.mean(x[0] for x in secs)
            unit = "steps/s" if args.config == 3 else "decodes/s"
            print(json.dumps({"impl": "reference", "metric": cfg["workload"], "value": 1.0 / t_unit, "unit": unit,
                              "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                              "ms_per_step": t_unit * 1e3, "higher_is_better": True, "scaling": "weak",
                              "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                              "config": {"workload": cfg["workload"]},
                              "extrapolated_from": "the 256^2 pass in `sample`, scaled by FLOPs: steps x "
                                                   "ms_per_step is not the time this run measured",
                              "cpu_baseline": {"value": 1.0 / t_unit, "unit": unit, "cores": secs[0][1],
                                               "kind": "port", "sample": secs[0][2]},
                              "e2e": {"value": 1.0 / t_unit, "unit": unit, "h2d_bytes_per_step": 0,
                                      "d2h_bytes_per_step": 0}}), flush=True)
    elif args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_mkb(args, cfg)


if __name__ == "__main__":
    main()
