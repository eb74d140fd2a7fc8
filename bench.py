#!/usr/bin/env python
"""Benchmark of the omni-tokenizer hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config NAME] [--items N]
                    [--rows N] [--impl ours|reference]

Default run: the headline is BASELINE config 2, the SigLIP-shaped encoder
self-attention op -- batch 32, 16 heads, L=729, head_dim 72, fp16 Q/K/V drawn
N(0,1)*0.5 from a seed -- the configuration BASELINE.json's metric
("attn TFLOP/s vs B200 BF16 peak") is quoted on.  One step = one attention
pass over that batch; FLOPs per step = 4*B*H*L^2*D (D = 72, not the padded 80).
The same line carries, under "sub", one record per other configuration the
metric names, each with its own roofline, cpu_baseline and e2e: c1 (Whisper
shape, bf16), c1_f32 (the same shape in fp32, the reference's audio profile),
c3 (variable-length audio batch), vq_audio and vq_image (the VQ argmin ops,
bf16 profile), vq_audio_f32 (the fp32-profile VQ at config 4's graph shape),
c5 (images/s of the whole image encoder), c4_bf16 and c4 (audio-s/s of the
whole audio encoder, bf16 mode and the fp32 profile).  --config NAME runs one configuration alone.

* value  -- device-resident inputs, K steps timed with CUDA events between a
            barrier + synchronize on both sides, max over ranks, whole job.
* e2e    -- the same metric through the C ABI host-buffer entry point
            (omni_b200_attention_bhld_host): every step copies Q/K/V from
            pinned host memory to the device and the output back.
* roofline -- algorithmic FLOPs per launch / mean kernel duration (CUDA events
            on the launching stream, measured in this run) vs the measured
            dense bf16 peak in MEASURED_PEAKS.json (fp32 inputs: that peak / 6,
            three tf32 products per fp32 product at half the bf16 rate).
* cpu_baseline -- the reference's own CPU attention (src/cpu.cpp compiled into
            oracle/_ref) on the host cores, on a bounded sample (rank 0, N=1).
Under torchrun (N > 1) the attention ops run one batch per rank (weak
scaling), except c3, whose one 64-segment batch is split into length-balanced
bins (strong scaling); the whole encoders split each step's items across
ranks (strong scaling).  No collective sits on the data path (timing uses one
all-reduce of a few scalars).

--impl reference times the reference's CPU implementation (oracle/_ref, or
the oracle port when the reference was not compiled here) on the same metric.

Whole encoders (c4, c4_bf16, c5; BASELINE configs 4 and 5): a seeded
random-weight OMNIVQ01 model of production shape is written per run and loaded
through the omni_* C ABI of libomni_b200.so; value = items/s (images/s, or
audio seconds/s) through the batched call on device-resident inputs, e2e = the
same call on host buffers; the CPU baseline is the reference's own CPU
library, extrapolated from 1- and 2-layer models.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    "c2": dict(kind="attn", B=32, H=16, L=729, D=72, dtype="f16", std=0.5, seed=1002,
               workload="SigLIP-shaped encoder self-attention op (BASELINE config 2)"),
    "c1": dict(kind="attn", B=1, H=20, L=1500, D=64, dtype="bf16", std=1.0, seed=1001,
               workload="Whisper-shaped encoder self-attention op (BASELINE config 1)"),
    "c1_f32": dict(kind="attn", B=1, H=20, L=1500, D=64, dtype="f32", std=1.0, seed=1001,
                   workload="Whisper-shaped encoder self-attention op (BASELINE config 1 shape) in fp32, the "
                            "reference's audio-profile precision: split-precision (3 x tf32) tensor-core kernel"),
    "c4_attn_f32": dict(kind="attn", B=16, H=16, L=1500, D=64, dtype="f32", std=1.0, seed=1004,
                        workload="attention of the fp32 audio encoder (BASELINE config 4 shape: 16 segments, "
                                 "16 heads, L 1500, head_dim 64), fp32 split-precision kernel"),
    "c3": dict(kind="attn", B=64, H=20, L=1500, D=64, dtype="bf16", std=1.0, seed=1003, varlen=(100, 1500),
               shard="balanced",
               workload="variable-length audio attention batch, key-padding mask (BASELINE config 3)"),
    "vq_audio": dict(kind="vq", N=24000, K=16384, dim=64, seed=1010,
                     workload="VQ argmin op, audio-shaped (x 24000x64 vs codebook 16384x64, bf16)"),
    "vq_image": dict(kind="vq", N=373248, K=16384, dim=32, seed=1011,
                     workload="VQ argmin op, image-shaped (x 373248x32 vs codebook 16384x32, bf16)"),
    # The fp32-profile VQ of BASELINE config 4's graph: 16 segments pool to
    # 16 x 188 rows of width 1024, searched against the 16384 x 1024 codebook.
    "vq_audio_f32": dict(kind="vq", N=3008, K=16384, dim=1024, profile="f32", seed=1012,
                         workload="VQ argmin op, fp32 profile at BASELINE config 4's graph shape (x 3008x1024 "
                                  "vs codebook 16384x1024: tf32 search, fp64 re-scoring of the candidates)"),
    # Whole encoders through the reference's omni_* C ABI (libomni_b200.so), on
    # randomly initialised OMNIVQ01 models of production shape.
    "c4": dict(kind="encoder", modality="audio", items=16, mel=80, frames=3000, width=1024, layers=24, heads=16,
               ffn=4096, positions=1500, block=1500, vocab=16384, seed=1004, audio_bf16=False,
               workload="full audio encoder (BASELINE config 4 body: 24 layers, d 1024, 16 heads, ffn 4096, "
                        "80 mel x 3000 frames; reference head: pool 4, fp32 VQ over 16384x1024; the reference's "
                        "fp32 audio profile)"),
    "c4_bf16": dict(kind="encoder", modality="audio", items=16, mel=80, frames=3000, width=1024, layers=24,
                    heads=16, ffn=4096, positions=1500, block=1500, vocab=16384, seed=1004, audio_bf16=True,
                    workload="full audio encoder, BASELINE config 4 precision (bf16 weights and activations, "
                             "fp32 LayerNorm statistics): this library's OMNI_B200_AUDIO_BF16=1 mode, same shapes "
                             "as c4"),
    # 378 = 27 x 14: the 27x27 patch grid a stride-14 conv takes from a 384x384
    # image; the reference ABI wants sides that are multiples of the patch.
    "c5": dict(kind="encoder", modality="image", items=512, size=378, patch=14, grid=27, width=1152, layers=27,
               heads=16, ffn=4304, code_dim=32, vocab=16384, seed=1005,
               workload="full image encoder (BASELINE config 5: 27 layers, d 1152, 16 heads of 72, ffn 4304, "
                        "729 patches of 14x14 (384x384 cropped to 378x378), 32-dim L2-normalised bf16 VQ "
                        "over 16384 codes)"),
}
METRIC = "attn TFLOP/s vs B200 BF16 peak"
L2_BYTES = 126 * 1024 * 1024


def load_package():
    import importlib.util

    name = "omni_tokenizer_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg = ROOT / "omni-tokenizer_b200"
    spec = importlib.util.spec_from_file_location(name, pkg / "__init__.py", submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    try:
        data = json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
        return data, "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML (read only)."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting",
               0x10: "sync_boost"}

    def __init__(self, cuda_index):
        self.samples = []
        self.ok = False
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            handle = None
            try:
                import torch

                props = torch.cuda.get_device_properties(cuda_index)
                bus = "%08x:%02x:%02x.0" % (props.pci_domain_id, props.pci_bus_id, props.pci_device_id)
                handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
            except Exception:
                handle = pynvml.nvmlDeviceGetHandleByIndex(cuda_index)
            self.h = handle
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None

    def _reasons(self):
        nv = self.nv
        fn = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or nv.nvmlDeviceGetCurrentClocksThrottleReasons
        return fn(self.h)

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                self.samples.append((time.perf_counter(), mhz, self._reasons()))
            except Exception:
                pass
            time.sleep(0.01)

    def start(self):
        if self.ok:
            self.thread = threading.Thread(target=self._run, daemon=True)
            self.thread.start()

    def stop(self):
        if self.ok:
            self._stop.set()
            self.thread.join()

    def summary(self, t0, t1):
        if not self.ok:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvml unavailable"], "samples": 0}
        inside = [s for s in self.samples if t0 <= s[0] <= t1]
        if not inside:  # a short region: take the samples nearest to it
            inside = sorted(self.samples, key=lambda s: min(abs(s[0] - t0), abs(s[0] - t1)))[:3]
        bits = 0
        for _, _, r in inside:
            bits |= r
        names = sorted({name for b, name in self.REASONS.items() if bits & b})
        return {"sm_mhz": statistics.median([s[1] for s in inside]) if inside else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(inside)}


# ------------------------------------------------------------------ inputs
def attn_inputs(cfg, rank, world=1):
    """Q, K, V (pinned host tensors) and the valid lengths of this rank's items.

    Weak-scaling configs give every rank its own seeded batch.  The sharded
    config (shard="balanced") draws one batch of B variable-length segments from
    its seed -- every segment from a generator of its own, so the data do not
    depend on the number of ranks -- and gives rank r the segments of bin r of
    sharding.balanced_bins (greedy longest-first by L^2)."""
    import torch

    B, H, L, D = cfg["B"], cfg["H"], cfg["L"], cfg["D"]
    dt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[cfg["dtype"]]
    if cfg.get("shard") == "balanced":
        lo, hi = cfg["varlen"]
        all_lengths = np.random.default_rng(cfg["seed"]).integers(lo, hi + 1, size=B).astype(np.int32)
        load_package()
        from omni_tokenizer_b200.sharding import balanced_bins

        mine = balanced_bins(all_lengths.tolist(), world)[rank]
        seg = []
        for i in mine:
            g = torch.Generator().manual_seed(cfg["seed"] * 1000 + i)
            seg.append([torch.randn(1, H, L, D, generator=g) * cfg["std"] for _ in range(3)])
        qkv = [torch.cat([s[j] for s in seg]).to(dt).pin_memory() for j in range(3)]
        return qkv, torch.from_numpy(all_lengths[mine].copy()), all_lengths
    g = torch.Generator().manual_seed(cfg["seed"] + 7919 * rank)
    qkv = [(torch.randn(B, H, L, D, generator=g) * cfg["std"]).to(dt).pin_memory() for _ in range(3)]
    lengths = None
    if cfg.get("varlen"):
        rng = np.random.default_rng(cfg["seed"] + 7919 * rank)
        lo, hi = cfg["varlen"]
        lengths = torch.from_numpy(rng.integers(lo, hi + 1, size=B).astype(np.int32))
    return qkv, lengths, None


def attn_flops(cfg, lengths, batch=None):
    """4 H D sum(L_i^2) over the items (valid query x valid key pairs for varlen)."""
    H, D, L = cfg["H"], cfg["D"], cfg["L"]
    if lengths is not None:
        lens = lengths.numpy() if hasattr(lengths, "numpy") else np.asarray(lengths)
        return 4.0 * H * D * float(np.sum(lens.astype(np.float64) ** 2))
    return 4.0 * (cfg["B"] if batch is None else batch) * H * L * L * D


def vq_inputs(cfg, rank):
    import torch

    g = torch.Generator().manual_seed(cfg["seed"] + 7919 * rank)
    dt = torch.float32 if cfg.get("profile") == "f32" else torch.bfloat16
    x = torch.randn(cfg["N"], cfg["dim"], generator=g).to(dt).pin_memory()
    cb = torch.randn(cfg["K"], cfg["dim"], generator=g).to(dt).pin_memory()
    return x, cb


# ------------------------------------------------------------------ CPU side
def cpu_reference_sample(cfg, budget_s, items=None):
    """Time the reference CPU attention / quantize on a bounded sample.

    Returns (flops_or_work, seconds, threads, kind, sample_text)."""
    from oracle import oracle as O

    kind = "reference" if O.ref_available() else "port"
    impl = "ref" if kind == "reference" else "oracle"
    threads = O.cpu_threads()
    rng = np.random.default_rng(cfg["seed"])
    if cfg["kind"] == "attn":
        H, L, D = cfg["H"], cfg["L"], cfg["D"]
        done_heads, flops, t_total = 0, 0.0, 0.0
        lengths = None
        if cfg.get("varlen"):
            lo, hi = cfg["varlen"]
            lengths = rng.integers(lo, hi + 1, size=cfg["B"])
        max_heads = cfg["B"] * H if items is None else items
        while done_heads < max_heads and (items is not None or t_total < budget_s or done_heads == 0):
            b = done_heads // H
            n = int(lengths[b]) if lengths is not None else L
            q = (rng.standard_normal((n, D)) * cfg["std"]).astype(np.float32)
            k = (rng.standard_normal((n, D)) * cfg["std"]).astype(np.float32)
            v = (rng.standard_normal((n, D)) * cfg["std"]).astype(np.float32)
            t0 = time.perf_counter()
            O.attention(q, k, v, 1, 0, n, False, False, impl=impl)
            t_total += time.perf_counter() - t0
            flops += 4.0 * n * n * D
            done_heads += 1
        sample = f"{done_heads} (item, head) slices of the workload, fp32, src/cpu.cpp Ops::attention"
        return flops, t_total, threads, kind, sample
    # VQ: a slice of rows against the full codebook.
    dim, K = cfg["dim"], cfg["K"]
    bf = cfg.get("profile") != "f32"
    rnd = O.round_bf16 if bf else (lambda a: a)
    cb = rnd(rng.standard_normal((K, dim)).astype(np.float32))
    norms = O.squares(cb, bf16=bf)
    rows, t_total, work = 64 if bf else 8, 0.0, 0.0
    done = chunks = 0
    while done < cfg["N"] and (chunks < items if items is not None else (t_total < budget_s or chunks == 0)):
        x = rnd(rng.standard_normal((rows, dim)).astype(np.float32))
        t0 = time.perf_counter()
        O.quantize(x, cb, norms, bf16=bf, impl=impl)
        t_total += time.perf_counter() - t0
        work += 2.0 * rows * K * dim
        done += rows
        chunks += 1
    return work, t_total, threads, kind, (f"{done} rows x {K} codes, {'bf16' if bf else 'fp32'} profile, "
                                          "src/cpu.cpp Ops::quantize")


# ------------------------------------------------------------------ whole encoders
def encoder_model_config(cfg, layers=None):
    load_package()
    import omni_tokenizer_b200.omnivq as ov

    n = cfg["layers"] if layers is None else layers
    if cfg["modality"] == "audio":
        return ov, ov.audio_config(layers=n, width=cfg["width"], heads=cfg["heads"], ffn=cfg["ffn"],
                                   mel=cfg["mel"], positions=cfg["positions"], block=cfg["block"],
                                   vocab=cfg["vocab"])
    return ov, ov.image_config(layers=n, width=cfg["width"], heads=cfg["heads"], ffn=cfg["ffn"],
                               patch=cfg["patch"], grid=cfg["grid"], code_dim=cfg["code_dim"], vocab=cfg["vocab"])


def encoder_flops(cfg, layers=None):
    """Algorithmic FLOPs of one item (one 30 s segment or one image): GEMM
    multiply-adds x 2 over the reference graph, attention 4 L^2 d per layer."""
    W, F = cfg["width"], cfg["ffn"]
    n = cfg["layers"] if layers is None else layers
    if cfg["modality"] == "audio":
        T = cfg["frames"]
        L = (T + 1) // 2
        stem = 2.0 * T * 3 * cfg["mel"] * W + 2.0 * L * 3 * W * W
        body = n * (2.0 * L * (4 * W * W + 2 * W * F) + 4.0 * L * L * W)
        vq = 2.0 * ((L + 3) // 4) * cfg["vocab"] * W
        return stem + body + vq
    g = cfg["size"] // cfg["patch"]
    L = g * g
    stem = 2.0 * L * 3 * cfg["patch"] ** 2 * W
    body = n * (2.0 * L * (4 * W * W + 2 * W * F) + 4.0 * L * L * W)
    head = 2.0 * L * W * cfg["code_dim"] + 2.0 * L * cfg["vocab"] * cfg["code_dim"]
    return stem + body + head


def encoder_inputs(cfg, count, seed):
    """U(-1, 1) log-mel segments [count, mel, frames] or images [count, 3, size, size]."""
    rng = np.random.default_rng(seed)
    if cfg["modality"] == "audio":
        shape = (count, cfg["mel"], cfg["frames"])
    else:
        shape = (count, 3, cfg["size"], cfg["size"])
    return rng.uniform(-1.0, 1.0, shape).astype(np.float32)


def encode_item(session, cfg, x):
    """One item through the reference's single-item call."""
    if cfg["modality"] == "audio":
        return session.encode_audio(x, cfg["frames"])
    return session.encode_image(x)


def encode_batch(session, cfg, x, device=None):
    """All items through the batched extension (host array, or a device tensor)."""
    shape = tuple(x.shape)
    ptr = None if device is None else device.data_ptr()
    if cfg["modality"] == "audio":
        valid = np.full(shape[0], cfg["frames"], np.uint32)
        return session.encode_audio_batch(x if ptr is None else shape, valid, device_ptr=ptr)
    return session.encode_images(x if ptr is None else shape, cfg["patch"], device_ptr=ptr)


def encoder_unit(cfg):
    return ("audio-s/s", 30.0 * cfg["frames"] / 3000) if cfg["modality"] == "audio" else ("images/s", 1.0)


def cpu_encoder_sample(cfg, tmpdir, repeats=1):
    """The reference's own CPU library (oracle/_ref/libomni_ref_full.so, all host
    threads) on 1- and 2-layer models of the workload's width, one item each;
    the per-item time of the full depth is extrapolated linearly in layers.
    Returns (seconds_per_item, threads, sample_text) or None without the library."""
    from oracle import oracle as O

    lib_path = ROOT / "oracle" / "_ref" / "libomni_ref_full.so"
    if not lib_path.is_file():
        return None
    load_package()
    import omni_tokenizer_b200.abi as abi

    ref = abi.OmniLib(lib_path)
    x = encoder_inputs(cfg, 1, cfg["seed"] + 99)[0]
    times = {}
    for n in (1, 2):
        ov, mc = encoder_model_config(cfg, layers=n)
        path = os.path.join(tmpdir, f"cpu_{cfg['modality']}_{n}.omni")
        ov.write_random_model(path, mc, seed=cfg["seed"] + n)
        with ref.load(path, backend=abi.CPU) as m:
            s = m.context()
            best = None
            for _ in range(repeats):
                t0 = time.perf_counter()
                encode_item(s, cfg, x)
                dt = time.perf_counter() - t0
                best = dt if best is None else min(best, dt)
            s.close()
        times[n] = best
        os.remove(path)
    per_layer = max(times[2] - times[1], 0.0)
    per_item = times[1] + (cfg["layers"] - 1) * per_layer
    sample = (f"1 item through 1- and 2-layer models of the same width on the reference CPU backend "
              f"({times[1]:.2f} s, {times[2]:.2f} s); per-item time extrapolated to {cfg['layers']} layers")
    return per_item, O.cpu_threads(), sample


def fp32_emulation_available():
    """Whether the cuBLAS bound in this process offers BF16x9 fp32 emulation."""
    import ctypes

    try:
        lib = ctypes.CDLL("libcublas.so.12", mode=os.RTLD_LAZY | os.RTLD_NOLOAD)
    except OSError:
        return False
    return hasattr(lib, "cublasSetEmulationStrategy")


def run_encoder_reference(args, cfg):
    """The reference arm of a whole-encoder config: its CPU library, rank 0 only."""
    import tempfile

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    unit_name, unit_per_item = encoder_unit(cfg)
    tmpdir = tempfile.mkdtemp(prefix="omni_bench_")
    # Each step is one item per model depth; the best of `steps` repeats counts.
    got = cpu_encoder_sample(cfg, tmpdir, repeats=max(1, min(args.steps, 3)))
    if got is None:
        return {"impl": "reference", "unavailable": "reference CPU library oracle/_ref/libomni_ref_full.so not built"}
    per_item, threads, sample = got
    value = unit_per_item / per_item
    return {
        "impl": "reference", "metric": f"{unit_name} (full encoder)", "value": value, "unit": unit_name,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * per_item * cfg["items"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32" if cfg["modality"] == "audio" else "bf16",
        "data": "synthetic (seeded U(-1,1) inputs, random-init weights)",
        "config": {"workload": cfg["workload"], "config": args.config, "items_per_step": cfg["items"],
                   "extrapolated": True},
        "cpu_baseline": {"value": value, "unit": unit_name, "cores": threads, "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": unit_name, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


_CPU_ENCODER_CACHE = {}


def run_encoder(args, name, cfg, dist, steps, warmup):
    """One whole-encoder config on this rank's share of the step's items
    (strong scaling).  Returns the JSON line on rank 0, None elsewhere."""
    import tempfile

    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    unit_name, unit_per_item = encoder_unit(cfg)
    flops_item = encoder_flops(cfg)
    tmpdir = tempfile.mkdtemp(prefix="omni_bench_")
    load_package()
    import omni_tokenizer_b200.abi as abi

    os.environ["OMNI_B200_AUDIO_BF16"] = "1" if cfg.get("audio_bf16") else "0"
    lib = abi.OmniLib(ROOT / "omni-tokenizer_b200" / "libomni_b200.so")
    emulated = fp32_emulation_available() and os.environ.get("OMNI_B200_FP32_EMULATION", "") != "0"
    # Every rank writes the same seeded model into its own temporary directory
    # (no shared filesystem is assumed between ranks).
    ov, mc = encoder_model_config(cfg)
    model_path = os.path.join(tmpdir, f"{name}.omni")
    t_write = time.perf_counter()
    ov.write_random_model(model_path, mc, seed=cfg["seed"])
    t_write = time.perf_counter() - t_write
    # Strong scaling: the step's items split evenly across ranks.
    share = [len(r) for r in np.array_split(np.arange(cfg["items"]), world)]
    mine = share[rank]
    # Host inputs live in pinned memory (the e2e leg copies them every step).
    host = torch.from_numpy(encoder_inputs(cfg, mine, cfg["seed"] + 7919 * rank)).pin_memory().numpy()
    dev = torch.from_numpy(host).cuda()

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    def timed(fn, n):
        barrier()
        t0 = time.perf_counter()
        out = 0
        for _ in range(n):
            out += fn().nbytes
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        barrier()
        return dt, out

    with lib.load(model_path, backend=abi.CUDA, device=local) as model:
        session = model.context()
        for _ in range(max(warmup, 3)):
            encode_batch(session, cfg, host, dev)
        sampler = ClockSampler(local)
        sampler.start()
        t_clock0 = time.perf_counter()
        # value: device-resident inputs through the batched extension.
        elapsed, _ = timed(lambda: encode_batch(session, cfg, host, dev), steps)
        t_clock1 = time.perf_counter()
        sampler.stop()
        # e2e: host buffers through the same call (host-to-device copies inside),
        # after two untimed calls: the first sizes the host path's staging
        # buffers, the second (the same key again) captures the call's CUDA graph,
        # which the timed calls replay (copies from the pinned inputs included).
        encode_batch(session, cfg, host)
        encode_batch(session, cfg, host)
        e2e_steps = max(1, min(steps, 3))
        e2e_elapsed, codes_bytes = timed(lambda: encode_batch(session, cfg, host), e2e_steps)
        # The reference's single-item calls on a sample of the rank's items (one
        # untimed call first, for the single-item shapes' buffers).
        sample = min(mine, 16 if cfg["modality"] == "image" else 4)
        encode_item(session, cfg, host[0])
        item_elapsed, _ = timed(lambda: np.concatenate([encode_item(session, cfg, x) for x in host[:sample]]), 1)
        # Kernel launches of one step, by name, through the profiler -- after the
        # timed regions: an attached profiler slows every later launch.
        launches_step, library_launches = None, None
        try:
            from torch.profiler import ProfilerActivity, profile

            with profile(activities=[ProfilerActivity.CUDA]) as prof:
                encode_batch(session, cfg, host, dev)
                torch.cuda.synchronize()
            names = [e.name for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA
                     and "memcpy" not in e.name.lower() and "memset" not in e.name.lower()]
            lib_like = ("gemm", "cutlass", "cublas", "nvjet", "xmma", "splitk", "reduce_1block", "inf_patching")
            library_launches = sum(1 for n in names if any(k in n.lower() for k in lib_like))
            launches_step = len(names) - library_launches
        except Exception:
            pass
        peak_ws = session.peak_workspace
        session.close()
    clocks = sampler.summary(t_clock0, t_clock1)
    os.remove(model_path)
    if dist is not None:
        t = torch.tensor([elapsed, e2e_elapsed, item_elapsed], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed, e2e_elapsed, item_elapsed = t.tolist()

    items_total = cfg["items"] * steps
    value = items_total * unit_per_item / elapsed
    e2e_value = cfg["items"] * e2e_steps * unit_per_item / e2e_elapsed
    per_item_value = sample * world * unit_per_item / item_elapsed
    tflops = items_total * flops_item / elapsed / 1e12 / world  # per GPU
    pk, pk_kind = peaks()
    peak = float(pk.get("bf16_tflops_sustained", pk.get("bf16_tflops", 1400.0)))
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        key = cfg["modality"]  # the reference's CPU profile: fp32 audio, bf16 image
        if key not in _CPU_ENCODER_CACHE:
            _CPU_ENCODER_CACHE[key] = cpu_encoder_sample(cfg, tmpdir)
        got = _CPU_ENCODER_CACHE[key]
        if got is not None:
            per_item, threads, sample_text = got
            cpu = {"value": unit_per_item / per_item, "unit": unit_name, "cores": threads, "kind": "reference",
                   "sample": sample_text + ("; the reference runs audio in fp32 only" if cfg.get("audio_bf16")
                                            else "")}
    in_item = int(np.prod(host.shape[1:])) * 4
    if rank != 0:
        return None
    return {
        "metric": f"{unit_name} (full encoder)",
        "value": value,
        "unit": unit_name,
        "n_gpus": world,
        "steps": steps,
        "warmup": max(warmup, 3),
        "ms_per_step": 1e3 * elapsed / steps,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32" if (cfg["modality"] == "audio" and not cfg.get("audio_bf16")) else "bf16",
        "data": "synthetic (seeded U(-1,1) inputs, random-init weights of the named shape)",
        "config": {
            "workload": cfg["workload"],
            "config": name,
            "items_per_step": cfg["items"],
            "items_per_rank": share,
            "flops_per_item": flops_item,
            "parallelism": f"item-sharded replicas x{world}" if world > 1 else "single GPU",
            "timing": "wall clock around the synchronous batched call omni_b200_encode_"
                      + ("audio_batch" if cfg["modality"] == "audio" else "images")
                      + " (device-resident inputs; codes copied back), synchronize + barrier on both sides, "
                        "max over ranks; e2e: the same call on pinned host buffers",
            "per_item_abi": {"value": per_item_value, "unit": unit_name, "items": sample,
                             "call": "omni_encode_" + cfg["modality"] + " (the reference's single-item call, "
                                     "host buffers)"},
            "fp32_gemms": ("BF16x9-emulated fp32 (cuBLAS)" if emulated else "fp32 on the CUDA cores")
                          if cfg["modality"] == "audio" and not cfg.get("audio_bf16") else None,
            "l2": "weights and activations far above L2 size per step; no flush",
            "model_write_s": round(t_write, 1),
            "peak_workspace_bytes": peak_ws,
        },
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": peak, "unit": "TFLOP/s",
                     "frac": tflops / peak, "traffic": None,
                     "peak_source": f"{pk_kind} bf16_tflops_sustained (whole-encoder FLOPs per GPU / wall time)"},
        "e2e": {"value": e2e_value, "unit": unit_name, "h2d_bytes_per_step": in_item * cfg["items"],
                "d2h_bytes_per_step": codes_bytes // e2e_steps * world},
        "cpu_baseline": cpu,
        "gpu_launches": None if launches_step is None else launches_step * steps,
        "library_launches": None if library_launches is None else library_launches * steps,
        "clocks": clocks,
    }


# ------------------------------------------------------------------ arms
def run_reference(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    # Size each step's sample so that warmup + steps end within ~2 minutes.
    probe_work, probe_t, threads, kind, _ = cpu_reference_sample(cfg, 0.0, items=1)
    per_unit = max(probe_t, 1e-4)
    budget = 120.0 / max(1, args.steps + args.warmup)
    vq_rows = 64 if cfg.get("profile") != "f32" else 8
    total_units = cfg["B"] * cfg["H"] if cfg["kind"] == "attn" else (cfg["N"] + vq_rows - 1) // vq_rows
    units = max(1, min(total_units, int(budget / per_unit)))
    for _ in range(args.warmup):
        cpu_reference_sample(cfg, 0.0, items=units)
    work, seconds = 0.0, 0.0
    for _ in range(args.steps):
        w, s, threads, kind, sample = cpu_reference_sample(cfg, 0.0, items=units)
        work += w
        seconds += s
    value = work / seconds / 1e12
    unit = "TFLOP/s"
    return {
        "impl": "reference", "metric": METRIC if cfg["kind"] == "attn" else "VQ TFLOP/s", "value": value,
        "unit": unit, "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * seconds / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": cfg["workload"], "sample_per_step": units},
        "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def e2e_timeline(ctx, e2e_step, in_bytes, out_bytes):
    """--e2e-timeline: the PCIe rates of this box for the step's byte counts
    (pinned buffers) and the CUDA activity of one end-to-end call, on stderr."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    def timed(fn, reps=10):
        fn()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(reps):
            fn()
        torch.cuda.synchronize()
        return (time.perf_counter() - t0) / reps

    hi, di = torch.empty(in_bytes, dtype=torch.uint8).pin_memory(), torch.empty(in_bytes, dtype=torch.uint8,
                                                                                   device="cuda")
    ho, do = torch.empty(out_bytes, dtype=torch.uint8).pin_memory(), torch.empty(out_bytes, dtype=torch.uint8,
                                                                                    device="cuda")
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()

    def both():
        with torch.cuda.stream(s_in):
            di.copy_(hi, non_blocking=True)
        with torch.cuda.stream(s_out):
            ho.copy_(do, non_blocking=True)

    t_in = timed(lambda: di.copy_(hi, non_blocking=True))
    t_out = timed(lambda: ho.copy_(do, non_blocking=True))
    t_both = timed(both)
    print(f"[e2e-timeline] H2D {in_bytes / 1e6:.1f} MB {t_in * 1e3:.3f} ms ({in_bytes / t_in / 1e9:.1f} GB/s); "
          f"D2H {out_bytes / 1e6:.1f} MB {t_out * 1e3:.3f} ms ({out_bytes / t_out / 1e9:.1f} GB/s); "
          f"both concurrently {t_both * 1e3:.3f} ms", file=sys.stderr)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        e2e_step(ctx)
        torch.cuda.synchronize()
    ev = sorted((e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA),
                key=lambda e: e.time_range.start)
    if ev:
        t0 = ev[0].time_range.start
        for e in ev:
            print(f"[e2e-timeline] {e.time_range.start - t0:9.1f} .. {e.time_range.end - t0:9.1f} us  "
                  f"{e.name[:60]}", file=sys.stderr)


def run_ours(args, name, cfg, dist, steps, warmup):
    """One op config (attention or VQ).  Returns the JSON line on rank 0."""
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    ob = load_package()
    lib = ob.library()
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    strong = cfg.get("shard") == "balanced"

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    if cfg["kind"] == "attn":
        (hq, hk, hv), lengths, all_lengths = attn_inputs(cfg, rank, world)
        q, k, v = (t.cuda() for t in (hq, hk, hv))
        out = torch.empty_like(q)
        dl = lengths.cuda() if lengths is not None else None
        B, H, L, D = q.shape
        dt = {"f16": 2, "bf16": 1, "f32": 0}[cfg["dtype"]]
        skip = 1 if lengths is not None else 0
        flops_step = attn_flops(cfg, lengths, batch=B)
        # Whole-job FLOPs of one step: every rank's batch (weak), or the one
        # sharded batch (strong).
        job_flops_step = attn_flops(cfg, all_lengths) if strong else flops_step * world
        launches_per_step = 1
        in_bytes = 3 * q.numel() * q.element_size()
        out_bytes = out.numel() * out.element_size()

        def step():
            lib.check(lib.lib.omni_b200_attention_bhld(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, H, L, D, dt, dt,
                dl.data_ptr() if dl is not None else None, 0, skip, 0.0, sp))

        hout = torch.empty_like(hq).pin_memory()
        hlen = lengths.numpy() if lengths is not None else None

        def e2e_step(ctx):
            ctx.attention_bhld(hq, hk, hv, hout, B, H, L, D, dt, dt, lengths=hlen, skip_padded_queries=skip)

        dtype_name = cfg["dtype"]
        working_set = in_bytes + out_bytes
    else:
        hx, hcb = vq_inputs(cfg, rank)
        x, cb = hx.cuda(), hcb.cuda()
        N, K, dim = cfg["N"], cfg["K"], cfg["dim"]
        prof = 0 if cfg.get("profile") == "f32" else 1  # OMNI_B200_F32 / OMNI_B200_BF16
        norms = torch.empty(K, dtype=x.dtype, device="cuda")
        lib.check(lib.lib.omni_b200_squares(cb.data_ptr(), norms.data_ptr(), K, dim, prof, prof, sp))
        ws_bytes = lib.lib.omni_b200_vq_workspace(N, dim, K, prof)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        ids = torch.empty(N, dtype=torch.int32, device="cuda")
        flops_step = 2.0 * N * K * dim
        job_flops_step = flops_step * world
        # bf16 dim <= 128: init, fused kernel, finish; wide or fp32: init, row
        # norms, one launch per pass, refinement (fp32).
        launches_per_step = 3 if (prof == 1 and dim <= 128) else (4 if prof == 1 else 6)

        def step():
            lib.check(lib.lib.omni_b200_vq_argmin(x.data_ptr(), cb.data_ptr(), norms.data_ptr(), ids.data_ptr(),
                                                  N, dim, K, prof, 0, ws.data_ptr(), ws_bytes, sp))

        hids = torch.empty(N, dtype=torch.int32).pin_memory()
        in_bytes = hx.numel() * hx.element_size() + hcb.numel() * hcb.element_size()
        out_bytes = N * 4

        def e2e_step(ctx):
            ctx.vq_argmin(hx, hcb, hids, N, dim, K, profile=prof, ids_u16=False)

        dtype_name = "f32" if prof == 0 else "bf16"
        working_set = in_bytes + out_bytes

    # ---- warm-up
    with torch.cuda.stream(stream):
        for _ in range(max(warmup, 3)):
            step()
    lib.sync_check(sp)

    sampler = ClockSampler(local)
    sampler.start()
    # ---- timed region (device-resident inputs)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    barrier()
    t_wall0 = time.perf_counter()
    with torch.cuda.stream(stream):
        ev[0].record(stream)
        for _ in range(steps):
            step()
        ev[1].record(stream)
    stream.synchronize()
    barrier()
    t_wall1 = time.perf_counter()
    lib.sync_check(sp)
    elapsed = ev[0].elapsed_time(ev[1]) / 1e3

    # ---- per-launch duration of the dominant kernel (events around single launches)
    pairs = []
    with torch.cuda.stream(stream):
        for _ in range(min(steps, 50)):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            step()
            b.record(stream)
            pairs.append((a, b))
    stream.synchronize()
    launch_s = statistics.mean(a.elapsed_time(b) for a, b in pairs) / 1e3
    sampler.stop()
    clocks = sampler.summary(t_wall0, t_wall1)

    # ---- end to end through the host-buffer C ABI
    e2e_steps = max(3, min(steps, 30))
    with ob.Context(local) as ctx:
        e2e_step(ctx)  # allocate buffers
        barrier()
        t0 = time.perf_counter()
        for _ in range(e2e_steps):
            e2e_step(ctx)
        e2e_elapsed = time.perf_counter() - t0
        if args.e2e_timeline and rank == 0:
            e2e_timeline(ctx, e2e_step, in_bytes, out_bytes)
    barrier()

    if dist is not None:
        t = torch.tensor([elapsed, e2e_elapsed / e2e_steps, launch_s], device="cuda", dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed, e2e_per_step, launch_s = t.tolist()
    else:
        e2e_per_step = e2e_elapsed / e2e_steps

    value = job_flops_step * steps / elapsed / 1e12
    e2e_value = job_flops_step / e2e_per_step / 1e12
    pk, pk_kind = peaks()
    peak = float(pk.get("bf16_tflops", 1590.0))
    peak_source = f"{pk_kind} bf16_tflops (burst)"
    if cfg.get("dtype") == "f32":
        # Three tf32 MMAs per fp32 product, tf32 at half the bf16 rate.
        peak /= 6.0
        peak_source = f"{pk_kind} bf16_tflops (burst) / 6: three tf32 products per fp32 product at half the bf16 rate"
    elif cfg.get("profile") == "f32":
        # The fp32 VQ's distance GEMM runs as kind::tf32 (half the bf16 rate).
        peak /= 2.0
        peak_source = f"{pk_kind} bf16_tflops (burst) / 2: the tf32 tensor rate of the distance search"
    achieved = flops_step / launch_s / 1e12
    traffic, traffic_source = None, None
    tf = ROOT / "profiles" / "traffic.json"
    if tf.is_file():
        try:
            rec = json.loads(tf.read_text()).get(name)
            if isinstance(rec, dict):
                traffic, traffic_source = rec.get("bytes"), rec.get("source")
        except Exception:
            traffic = None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        work, secs, threads, kind, sample = cpu_reference_sample(cfg, args.cpu_seconds)
        cpu = {"value": work / secs / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": kind, "sample": sample}

    if rank != 0:
        return None
    return {
        "metric": METRIC if cfg["kind"] == "attn" else "VQ TFLOP/s (distance GEMM + argmin)",
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": max(warmup, 3),
        "ms_per_step": 1e3 * elapsed / steps,
        "higher_is_better": True,
        "scaling": "strong" if strong else "weak",
        "vs_baseline": None,
        "dtype": dtype_name,
        "data": "synthetic (seeded, BASELINE shapes)",
        "config": {
            "workload": cfg["workload"],
            "config": name,
            "per_gpu_flops_per_step": flops_step,
            "job_flops_per_step": job_flops_step,
            "parallelism": (f"one batch sharded over {world} ranks by length-balanced bins" if strong else
                            f"item-sharded replicas x{world}") if world > 1 else "single GPU",
            "l2": f"working set {working_set / 2**20:.0f} MiB vs 126 MiB L2, no flush"
                  if working_set > L2_BYTES else "working set below L2 size: L2-resident between steps",
        },
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": traffic, "traffic_source": traffic_source,
                     "peak_source": peak_source},
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "h2d_bytes_per_step": in_bytes,
                "d2h_bytes_per_step": out_bytes},
        "cpu_baseline": cpu,
        "gpu_launches": launches_per_step * steps,
        "clocks": clocks,
    }


# Sub-records of the default run: the other BASELINE configurations the metric
# names (attention at the other shapes; images/s and audio-s/s of the whole
# encoders), each with its own roofline, cpu_baseline and e2e.
SUITE = ["c1", "c1_f32", "c3", "vq_audio", "vq_image", "vq_audio_f32", "c5", "c4_bf16", "c4"]
ENCODER_MAX_STEPS = 5


def run_config(args, name, dist, steps, warmup):
    cfg = dict(CONFIGS[name])
    if cfg["kind"] == "vq" and args.rows is not None and name == args.config:
        cfg["N"] = args.rows
    if cfg["kind"] == "encoder":
        if args.items is not None and name == args.config:
            cfg["items"] = args.items
        return run_encoder(args, name, cfg, dist, steps, warmup)
    return run_ours(args, name, cfg, dist, steps, warmup)


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--config", default=None, choices=sorted(CONFIGS),
                    help="run one configuration (default: c2 as the headline, the others as sub-records)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-seconds", type=float, default=5.0, help="CPU baseline sample budget")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub", action="store_true", help="default run: the headline line only")
    ap.add_argument("--items", type=int, default=None,
                    help="whole-encoder configs: items per step (default: the config's; smaller for profiling)")
    ap.add_argument("--e2e-timeline", action="store_true",
                    help="op configs: print the PCIe rates and the CUDA timeline of one end-to-end call (stderr)")
    ap.add_argument("--rows", type=int, default=None,
                    help="VQ configs: rows of x (default: the config's; smaller for profiling)")
    args = ap.parse_args()
    if args.rows is not None and (args.config is None or CONFIGS[args.config]["kind"] != "vq" or args.rows <= 0):
        ap.error("--rows applies to an explicit VQ --config and must be positive")
    if args.items is not None and (args.config is None or CONFIGS[args.config]["kind"] != "encoder"
                                   or args.items <= 0):
        ap.error("--items applies to an explicit whole-encoder --config and must be positive")
    if args.impl == "reference":
        cfg = dict(CONFIGS[args.config or "c2"])
        if cfg["kind"] == "encoder":
            line = run_encoder_reference(args, cfg)
        else:
            line = run_reference(args, cfg)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0
    # This library loads before torch, so that its cuBLAS (the toolkit's, with
    # fp32 emulation) is the one the process binds rather than torch's older copy.
    load_package().library()
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local))
    try:
        if args.config is not None:
            line = run_config(args, args.config, dist, args.steps, args.warmup)
        else:
            line = run_config(args, "c2", dist, args.steps, args.warmup)
            if not args.no_sub:
                subs = {}
                for name in SUITE:
                    enc = CONFIGS[name]["kind"] == "encoder"
                    sub = run_config(args, name, dist, min(args.steps, ENCODER_MAX_STEPS) if enc else args.steps,
                                     min(args.warmup, 3) if enc else args.warmup)
                    if sub is not None:
                        subs[name] = sub
                if line is not None:
                    line["sub"] = subs
        if line is not None:
            print(json.dumps(line), flush=True)
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
