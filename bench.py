"""Benchmark: ThetaScan mixer forward+backward tokens/s on B200.

Default workload (N=1): config 2 of the baseline -- kernel family, ReLU^2
ridge features, m = 256 from 2x random feature expansion, partial RoPE, a
one-branch fast recency bank with per-head alpha ~ U(0.9, 0.999), output gate,
B=8, T=4096, d_model=1024, H=16, d=64, bf16 activations with f32 state.
A step is one forward + backward of the whole mixer (projections included)
on synthetic x ~ N(0,1) with loss = mean(y^2).

With --gpus N (torchrun, one rank per GPU) every rank runs its own batch of
the same shape (weak scaling: independent (batch, head) units) and the ranks
all-reduce the mixer's parameter gradients over NCCL, as a data-parallel
step does.  ``--config c4`` (config 4: T = 32768, B-spline features, four
views) instead splits the sequences into N contiguous shards, one per rank,
that exchange their chunk states with one NCCL all-gather per step (strong
scaling: the B x T tokens are fixed).  ``--impl reference`` times the reference package's own CPU
implementation (its chunk backend, float32, from ``baseline/_ref``) on the host cores.

One JSON line is printed by rank 0.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

METRIC = "mixer fwd+bwd tokens/s at T=4K/32K, 1/2/4/8 B200, % of tensor roofline"
CONFIGS = {
    # name: (B, T, d_model, H, memory_multiplier, expansion, feature_map, rope, J)
    "c2": dict(B=8, T=4096, D=1024, H=16, mult=4, expansion=2, fmap="relu2_ridge", rope="partial", J=1),
    # config 1: the reference's float32 case (softmax partition, m = d = 64, recency
    # bank initialised at 0.95), float32 end to end on the f32 scan kernels
    "c1": dict(B=2, T=512, D=256, H=4, mult=1, expansion=1, fmap="softmax_partition", rope="none", J=1,
               dtype="f32", retention_spread=False),
    "small": dict(B=2, T=1024, D=512, H=8, mult=4, expansion=2, fmap="relu2_ridge", rope="partial", J=1),
    # config-2 shapes at batch 2: inputs still larger than L2, for profiler captures
    "c2b2": dict(B=2, T=4096, D=1024, H=16, mult=4, expansion=2, fmap="relu2_ridge", rope="partial", J=1),
    # config 4 at batch 1 (profiling captures of its tile kernels)
    "c4b1": dict(B=1, T=32768, D=1024, H=16, mult=2, expansion=1, fmap="projected_bspline", basis=16,
                 rope="partial", J=3, retentions=(0.9, 0.99, 0.999)),
    # config 4: B-spline features (16 basis functions, m = 2d = 128, P = 8
    # projections), bank of three recency branches 0.9 / 0.99 / 0.999 plus the
    # sum view; with --gpus N the 32K-token sequences are split into N shards.
    "c4": dict(B=4, T=32768, D=1024, H=16, mult=2, expansion=1, fmap="projected_bspline", basis=16,
               rope="partial", J=3, retentions=(0.9, 0.99, 0.999), seqpar=True),
    # config 3: Gauss-Newton fast weights, head_dim 128, m = 128, relu2, two-stage
    # feature-mass read (both_feature_mass), one Jacobian step, the plain sum view.
    # The reference rejects a feature-mass read normalisation for any net but
    # relu2 / relu2_threshold (config.py:85-90), so config 3's "tanh with read
    # normalisation on" runs as relu2 here; the tanh net (with damping) is
    # checked for parity with the read normalisation off.
    # config 5: a ~17M-parameter hybrid LM training step (nine blocks, d_model
    # 512, 8 heads, vocab 1024, tied embeddings, MLP ratio 2; the two middle
    # blocks ThetaScan-GN with 2x expansion, the rest causal attention),
    # global batch 64 x 1024 uniform token ids, AdamW, bf16 autocast; the
    # global batch is split over the GPUs (strong scaling).
    "c5": dict(B=64, T=1024, D=512, H=8, vocab=1024, layers=9, family="lm"),
    "c3": dict(B=8, T=8192, D=1024, H=8, mult=1, expansion=1, family="gn", fmap="relu2",
               gn_read="both_feature_mass", rope="partial", J=0),
}

WORKLOADS = {
    "c1": "config 1: ThetaScan-Kernel softmax partition m=64, fast bank 0.95, output gate, float32 end to end "
          "(float32 scan kernels on the CUDA cores); fwd+bwd, loss=mean(y^2)",
    "c2": "config 2: ThetaScan-Kernel relu2 ridge m=256 (2x expansion), partial RoPE, 1-branch fast bank, "
          "output gate; fwd+bwd, loss=mean(y^2)",
    "c3": "config 3: ThetaScan-GN relu2, head_dim 128, m=128, two-stage feature-mass read "
          "(both_feature_mass), 1 Jacobian step, sum view, output gate; fwd+bwd, loss=mean(y^2)",
    "c5": "config 5: hybrid LM training step, 9 blocks (d_model 512, 8 heads, MLP ratio 2, vocab 1024, tied "
          "embeddings), blocks 4-5 ThetaScan-GN (relu2 threshold, 2x expansion, m=256, two-stage feature-mass "
          "read, fast bank), the rest causal attention; global batch 64 x 1024 uniform tokens, AdamW, bf16 "
          "autocast",
    "c4": "config 4: ThetaScan-Kernel projected B-spline (16 basis, m=128), partial RoPE, fast bank "
          "0.9/0.99/0.999 + sum (4 views), output gate, T=32768; sequence-sharded over the GPUs; "
          "fwd+bwd, loss=mean(y^2)",
}


# --------------------------------------------------------------------------- workload

def build_module(cfg, device):
    from thetascan_b200.config import GNConfig, KernelConfig, RoPEConfig, TemporalConfig, ThetaScanConfig
    from thetascan_b200.mixer import ThetaScan
    if cfg.get("family") == "gn":
        config = ThetaScanConfig(
            d_model=cfg["D"], n_heads=cfg["H"], memory_multiplier=cfg["mult"], family="gn",
            gn=GNConfig(nonlinearity=cfg["fmap"], jacobian_steps=1, read_normalization=cfg["gn_read"]),
            rope=RoPEConfig(mode=cfg["rope"], fraction=0.5), temporal=TemporalConfig(mode="sum"))
        torch.manual_seed(0)
        module = ThetaScan(config)
        with torch.no_grad():
            module._core.W2[0].normal_(0.0, 0.02)   # a trained-like slow W2 (zero-init makes the write trivial)
        return module.to(device), config
    kernel = KernelConfig(feature_map=cfg["fmap"], bspline_basis_count=cfg.get("basis", 8))
    if cfg["J"] == 1:
        temporal = TemporalConfig(mode="bank", retention_init=0.95)
    else:
        temporal = TemporalConfig(mode="bank", recency_branches=cfg["J"], retention_inits=cfg["retentions"])
    config = ThetaScanConfig(
        d_model=cfg["D"], n_heads=cfg["H"], memory_multiplier=cfg["mult"], feature_expansion=cfg["expansion"],
        family="kernel", kernel=kernel, rope=RoPEConfig(mode=cfg["rope"], fraction=0.5), temporal=temporal)
    torch.manual_seed(0)
    module = ThetaScan(config)
    if cfg["J"] == 1 and cfg.get("retention_spread", True):
        # per-head retentions alpha_h ~ U(0.9, 0.999), as the config-2 statement has them
        with torch.no_grad():
            alphas = 0.9 + 0.099 * torch.rand(cfg["H"], generator=torch.Generator().manual_seed(0))
            module._core.fade_alpha.copy_(torch.log(alphas / (1.0 - alphas)))
    return module.to(device), config


def flops_per_token(cfg):
    """Algorithmic FLOPs per token, forward+backward (= 3x forward).

    Fixed counting convention: reference chunk C=64 with causal-half score,
    elementwise work counted as zero.  Returns (core, full mixer, per-phase
    forward FLOPs per token)."""
    H, d = cfg["H"], cfg["D"] // cfg["H"]
    m = cfg["mult"] * d
    C, V = 64, 1 + cfg["J"]
    if cfg.get("family") == "gn":
        # GN both_feature_mass: write 10 m d (W1 k, W2 h, W2^2 s^2, W2^T lambda; read W1 q),
        # stage 1 and stage 2 scans per view, and the stage-2 slow decode 2 d m
        feature = 10 * m * d
        scan = C * m + V * (C * (m + 1) + 4 * m * (m + 1) + 2 * d * m + C * m + C * (d + 1) + 4 * m * (d + 1))
    else:
        P = m // cfg["basis"] if cfg["fmap"] == "projected_bspline" else m
        feature = 4 * P * d + 2 * d * m
        scan = C * m + V * (C * (d + 1) + 4 * m * (d + 1))
    D, Hd = cfg["D"], H * d
    proj = 2 * D * 3 * Hd + 2 * Hd * D + 2 * D * Hd
    core = 3 * H * (feature + scan)
    return core, core + 3 * proj, {"feature": H * feature, "scan": H * scan}


# --------------------------------------------------------------------------- measurement helpers

class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled during the timed region.

    A thread reads NVML every 10 ms (read-only queries: the current and the
    maximum SM clock and the active clock-event reasons); where NVML cannot be
    loaded it reads ``nvidia-smi -lms 200`` instead.  ``__enter__`` returns once
    the first sample is in, so that the record covers the start of the timed
    region as well as its end."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown"),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown"),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown"),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap"))

    def __init__(self, bus_id, period_s=0.01):
        # The device is named by its PCI bus id ("DDDDDDDD:BB:DD.F"), not an
        # ordinal: NVML and nvidia-smi number GPUs physically and ignore
        # CUDA_VISIBLE_DEVICES, so the CUDA ordinal of a leased GPU can be
        # another GPU's NVML index.
        self.bus_id = bus_id
        self.period = period_s
        self.proc = None
        self.thread = None
        self.stop = threading.Event()
        self.samples = []  # (sm MHz, max sm MHz, set of active reasons)
        self.source = None

    def __enter__(self):
        if not self._start_nvml():
            self._start_smi()
        deadline = time.perf_counter() + 3.0
        while (not self.samples and self.thread is not None and self.thread.is_alive()
               and time.perf_counter() < deadline):
            time.sleep(0.002)
        return self

    def _start_nvml(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            by_bus = getattr(pynvml, "nvmlDeviceGetHandleByPciBusId_v2", None) or \
                pynvml.nvmlDeviceGetHandleByPciBusId
            handle = by_bus(self.bus_id)
            max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM))
            masks = [(name, getattr(pynvml, attr)) for name, attr in self.REASONS]

            def sample():
                sm = float(pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM))
                bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle)
                return sm, max_mhz, {name for name, mask in masks if bits & mask}

            first = sample()
        except Exception:
            return False

        def run():
            try:
                self.samples.append(first)
                while not self.stop.wait(self.period):
                    self.samples.append(sample())
            except Exception:
                pass
            finally:
                try:
                    pynvml.nvmlShutdown()
                except Exception:
                    pass

        self.source = f"nvml every {self.period * 1e3:.0f} ms"
        self.thread = threading.Thread(target=run, daemon=True)
        self.thread.start()
        return True

    def _start_smi(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self.bus_id, f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.source = "nvidia-smi every 200 ms"
        self.thread = threading.Thread(target=self._read_smi, daemon=True)
        self.thread.start()

    def _read_smi(self):
        names = [name for name, _ in self.REASONS]
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm, mx = float(parts[1]), float(parts[2])
            except ValueError:
                continue
            self.samples.append((sm, mx, {n for n, flag in zip(names, parts[5:9])
                                          if flag.lower().startswith("active")}))

    def __exit__(self, *exc):
        self.stop.set()
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)

    def summary(self):
        samples = list(self.samples)
        if not samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "bus_id": self.bus_id}
        return {"sm_mhz": statistics.median(s[0] for s in samples),
                "sm_max_mhz": max(s[1] for s in samples),
                "reasons": sorted(set().union(*(s[2] for s in samples))),
                "samples": len(samples), "sampler": self.source, "bus_id": self.bus_id}


def device_bus_id(index):
    """PCI bus id of CUDA device ``index`` in NVML's format."""
    props = torch.cuda.get_device_properties(index)
    return f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"


class PhaseTimer:
    """Time each C-ABI entry point with CUDA events on the launching stream
    (wraps the bound ctypes functions of the library)."""

    ENTRY_POINTS = ("ts_b200_feature_fwd", "ts_b200_scan_fwd", "ts_b200_kread_fwd", "ts_b200_kread_bwd",
                    "ts_b200_scan_bwd", "ts_b200_feature_bwd")

    def __init__(self, lib):
        self.lib = lib
        self.saved = {}
        self.events = {name: [] for name in self.ENTRY_POINTS}
        self.timing = False

    def install(self):
        for name in self.ENTRY_POINTS:
            fn = getattr(self.lib, name)
            self.saved[name] = fn

            def wrapper(*a, _fn=fn, _name=name):
                if not self.timing:
                    return _fn(*a)
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
                rc = _fn(*a)
                end.record()
                self.events[_name].append((start, end))
                return rc
            setattr(self.lib, name, wrapper)

    def uninstall(self):
        for name, fn in self.saved.items():
            setattr(self.lib, name, fn)

    def total_ms(self):
        """Device time of each entry point summed over the timed calls (a
        sequence shard calls the scan entry points twice per step)."""
        torch.cuda.synchronize()
        return {n: sum(s.elapsed_time(e) for s, e in ev) for n, ev in self.events.items() if ev}


def load_peaks():
    """(sustained bf16 TFLOP/s, burst bf16 TFLOP/s, HBM GB/s, source)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            peaks = json.load(f)
        return (peaks.get("bf16_tflops_sustained", 1403.9), peaks.get("bf16_tflops", 1638.2),
                peaks.get("hbm_gbs", 6650.0), "measured")
    return 1400.0, 1590.0, 6650.0, "fallback"


def bytes_per_token(cfg):
    """Compulsory HBM bytes per token of each entry point: its inputs read and
    outputs written once (bf16 streams, f32 reads / y0; chunk states and other
    scratch excluded).  Per head: x = d-wide q/k rows, m-wide features, R
    retention slots of width d+2 ([N | D | D], the mass column twice)."""
    H, d = cfg["H"], cfg["D"] // cfg["H"]
    m = cfg["mult"] * d
    R = 1 + cfg["J"]
    if cfg.get("family") == "gn":
        # stage 1: h0, h, g in, [g|1] f32 out; stage 2: h_q, h, lambda in, [lambda|1] f32 out
        fwd = H * R * ((3 * m) * 2 + (m + 1) * 4 + (2 * m + d) * 2 + (d + 1) * 4)
        return {"ts_b200_scan_fwd": fwd, "ts_b200_scan_bwd": 2 * fwd}
    return {
        "ts_b200_feature_fwd": H * (2 * d * 2 + 2 * m * 2 + d * 4),               # q,k in; phi q,k, y0 out
        "ts_b200_feature_bwd": H * (2 * d * 2 + 2 * m * 2 + d * 2 + 2 * d * 2),   # q,k, dphi q,k, dy in; dq,dk out
        "ts_b200_scan_fwd": H * (2 * m * 2 + d * 2 + R * (d + 2) * 4),            # phi q,k, v in; slots out
        "ts_b200_scan_bwd": H * (2 * m * 2 + d * 2 + R * (d + 2) * 2 + 2 * m * 2 + d * 2),
        "ts_b200_kread_fwd": H * (R * (d + 2) * 4 + d * 4 + d * 2),
        "ts_b200_kread_bwd": H * (R * (d + 2) * 4 + d * 2 + R * (d + 2) * 2),
    }


def source_hash():
    """First 16 hex digits of a SHA-256 over the library's sources (the CUDA
    files and the C-ABI header), naming the build a profile was taken on."""
    import hashlib
    h = hashlib.sha256()
    names = sorted(os.listdir(os.path.join(ROOT, "thetascan_b200", "csrc")))
    for name in names:
        with open(os.path.join(ROOT, "thetascan_b200", "csrc", name), "rb") as f:
            h.update(name.encode() + b"\0" + f.read())
    with open(os.path.join(ROOT, "include", "thetascan_b200.h"), "rb") as f:
        h.update(f.read())
    return h.hexdigest()[:16]


def measured_traffic(entry, tokens):
    """DRAM bytes (read + write) of one launch of a C-ABI entry point, from
    the ncu summary ``profiles/traffic_c2.md``: its kernels' bytes at the
    profiled size, scaled by tokens to this launch (traffic grows with
    B * T), and only when the summary names this build's source hash
    (``None`` otherwise, so a stale profile never reports)."""
    path = os.path.join(ROOT, "profiles", "traffic_c2.md")
    if not os.path.exists(path):
        return None, "no traffic profile"
    rows, build, tokens_at = {}, None, None
    with open(path) as f:
        for line in f:
            if line.startswith("source hash:"):
                build = line.split(":", 1)[1].strip().strip("`")
            elif line.startswith("tokens per launch:"):
                tokens_at = int(line.split(":", 1)[1])
            elif line.startswith("| `ts_b200_"):
                cells = [c.strip().strip("`") for c in line.strip().strip("|").split("|")]
                rows[cells[0]] = float(cells[1]) * 1e6
    if build != source_hash():
        return None, f"profile of build {build}, this build is {source_hash()}"
    if entry not in rows or not tokens_at:
        return None, "entry point not profiled"
    return rows[entry] * tokens / tokens_at, f"profiles/traffic_c2.md (build {build})"


# --------------------------------------------------------------------------- CPU reference

def reference_package():
    """The reference ``thetascan`` package itself (pure PyTorch): the
    directory ``$THETASCAN_REFERENCE_PATH`` names, else the offline install
    under ``baseline/_ref``; None where neither holds it."""
    path = os.environ.get("THETASCAN_REFERENCE_PATH") or os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(path, "thetascan")):
        return None
    if path not in sys.path:
        sys.path.insert(0, path)
    import thetascan
    return thetascan


def reference_module(ts, cfg, backend, view_set):
    """The reference's own public mixer for a bench workload, float32 on the
    CPU, with ``backend`` ("chunk", its fastest CPU path, or "cumsum", which
    takes the plain sum view only) and the same seeded weights as the GPU
    arm's module.  A bank of more than two recency branches (config 4) is
    beyond the reference's configuration; its arm runs two (0.9, 0.99)."""
    C = ts
    runtime = C.RuntimeConfig(backend=backend)
    if cfg.get("family") == "gn":
        config = C.ThetaScanConfig(
            d_model=cfg["D"], n_heads=cfg["H"], memory_multiplier=cfg["mult"], family="gn",
            gn=C.GNConfig(nonlinearity=cfg["fmap"], jacobian_steps=1, read_normalization=cfg["gn_read"]),
            rope=C.RoPEConfig(mode=cfg["rope"], fraction=0.5), temporal=C.TemporalConfig(mode="sum"),
            runtime=runtime)
    else:
        kernel = C.KernelConfig(feature_map=cfg["fmap"], bspline_basis_count=cfg.get("basis", 8))
        if view_set == "sum":
            temporal = C.TemporalConfig(mode="sum")
        elif cfg["J"] == 1:
            temporal = C.TemporalConfig(mode="bank", retention_init=0.95)
        else:
            temporal = C.TemporalConfig(mode="bank", recency_branches=2, retention_inits=tuple(cfg["retentions"][:2]))
        config = C.ThetaScanConfig(
            d_model=cfg["D"], n_heads=cfg["H"], memory_multiplier=cfg["mult"],
            feature_expansion=cfg["expansion"], family="kernel", kernel=kernel,
            rope=C.RoPEConfig(mode=cfg["rope"], fraction=0.5), temporal=temporal, runtime=runtime)
    torch.manual_seed(0)
    module = C.ThetaScan(config).float()
    if view_set != "sum" and cfg.get("family") != "gn" and cfg["J"] == 1 and cfg.get("retention_spread", True):
        with torch.no_grad():
            alphas = 0.9 + 0.099 * torch.rand(cfg["H"], generator=torch.Generator().manual_seed(0))
            module._core.fade_alpha.copy_(torch.log(alphas / (1.0 - alphas)))
    return module


def cpu_reference_step(cfg, T, view_set):
    """One forward+backward on the host CPU of the reference's own code for
    this workload at batch 1 and ``T`` tokens; returns (seconds, kind).

    ``view_set="bank"`` runs the reference's chunk backend with the
    workload's bank (its fastest CPU path); ``"sum"`` runs its cumsum backend,
    which the reference restricts to the plain sum view.  Where the reference
    package is absent, the float32 restatement under ``oracle/`` runs the same
    algorithm instead (kind "port")."""
    ts = reference_package()
    x = torch.randn(1, T, cfg["D"], generator=torch.Generator().manual_seed(0))
    if ts is not None:
        module = reference_module(ts, cfg, "cumsum" if view_set == "sum" else "chunk", view_set)
        t0 = time.perf_counter()
        y = module(x)
        y.square().mean().backward()
        return time.perf_counter() - t0, "reference"
    from oracle import mixer as omixer
    from oracle import scan as oscan

    module, _ = build_module(cfg, torch.device("cpu"))
    params = {n: t.detach().float().requires_grad_(True) for n, t in module._core.named_parameters()}
    for n, t in module._core.named_buffers():
        if n.startswith("_expand_"):
            params[n] = t.float()
    d = cfg["D"] // cfg["H"]
    core_cfg = {"n_heads": cfg["H"], "head_dim": d, "feature_expansion": cfg["expansion"],
                "kernel_kind": cfg["fmap"], "rope": cfg["rope"], "rope_frac": 0.5, "rope_base": 10000.0,
                "read_fade": view_set == "bank", "read_fade_mode": "fast", "read_norm": "key_mass", "eps": 1e-6,
                "scan_chunk": 512}
    if view_set == "sum":
        scan_fn = lambda q, k, v, rets: tuple(oscan.linattn_cumsum(q, k, v) for _ in rets)
    else:
        scan_fn = None
    t0 = time.perf_counter()
    y = omixer.mixer_forward(params, core_cfg, x, scan_fn=scan_fn)
    y.square().mean().backward()
    return time.perf_counter() - t0, "port"


def _reference_sample(kind, view_set, T, n):
    what = ("the reference package's chunk backend (its fastest CPU path), the workload's view bank"
            if view_set == "bank" else
            "the reference package's cumsum backend, plain sum view (cumsum rejects banks)")
    if kind == "port":
        what = "float32 restatement of the reference under oracle/ (reference package absent): " + what
    return (f"{what}; float32, batch 1 x {T} tokens of the workload's per-token shape, forward+backward, "
            f"median of {n}; tokens/s = {T} / median seconds (the GPU arm's batch and length are larger)")


def reference_lm_step(cfg, T):
    """One training step (forward, backward, AdamW) of the config-5 hybrid LM
    on the host CPU with the reference package's own GN mixer (float32,
    chunk backend), batch 1 x T tokens; returns (seconds, kind)."""
    from thetascan_b200.lm import HybridLM, gn_mixer_config
    ts = reference_package()
    if ts is None:
        raise SystemExit("config 5's reference arm needs the reference package (baseline/_ref)")

    def reference_mixer(c):
        d = c.to_dict()
        d["gn"] = {k: v for k, v in d["gn"].items() if k != "damping"}
        d["runtime"] = {"backend": "chunk", "scan_chunk": 512}
        return ts.ThetaScan(ts.ThetaScanConfig.from_dict(d))

    torch.manual_seed(2)
    model = HybridLM(vocab=cfg["vocab"], d_model=cfg["D"], n_layers=cfg["layers"], n_heads=cfg["H"],
                     mixer_config=gn_mixer_config(cfg["D"], cfg["H"]), mixer_factory=reference_mixer)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, weight_decay=0.0)
    tokens = torch.randint(0, cfg["vocab"], (1, T + 1), generator=torch.Generator().manual_seed(2))
    t0 = time.perf_counter()
    model.loss(tokens).backward()
    opt.step()
    return time.perf_counter() - t0, "reference"


def run_reference(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    T = args.ref_tokens
    if cfg.get("family") == "lm":
        for _ in range(args.warmup):
            reference_lm_step(cfg, T)
        runs = [reference_lm_step(cfg, T) for _ in range(max(1, args.steps))]
        per_step = statistics.median(t for t, _ in runs)
        value = T / per_step
        sample = (f"the config-5 hybrid LM on the host CPU with the reference package's own GN mixer (chunk "
                  f"backend), float32, batch 1 x {T} tokens, forward+backward+AdamW, median of {len(runs)}; "
                  f"tokens/s = {T} / median seconds")
        print(json.dumps({
            "impl": "reference", "metric": "hybrid LM training step tokens/s (config 5)", "value": value,
            "unit": "tokens/s", "n_gpus": args.gpus, "steps": len(runs), "warmup": args.warmup,
            "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"c5 bounded CPU sample B=1 T={T}", "model": "hybrid LM (reference mixer)",
                       "global_batch": 1, "seq_len": T, "parallelism": "cpu"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "reference",
                             "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
            flush=True)
        return
    for _ in range(args.warmup):              # untimed warm-up steps of the same sample
        cpu_reference_step(cfg, T, "bank")
    runs = [cpu_reference_step(cfg, T, "bank") for _ in range(max(1, args.steps))]
    per_step = statistics.median(t for t, _ in runs)
    kind = runs[0][1]
    value = T / per_step
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": len(runs), "warmup": args.warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{args.config} per-token shape, bounded CPU sample B=1 T={T}",
                   "model": "ThetaScan mixer (reference package)", "global_batch": 1, "seq_len": T,
                   "parallelism": "cpu", "normalization": "tokens/s = B*T of the sample / seconds per step"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": kind,
                         "sample": _reference_sample(kind, "bank", T, len(runs))},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- GPU arm

def run_b200(args, cfg):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120))
    device = torch.device("cuda", local)
    from thetascan_b200 import _lib

    module, config = build_module(cfg, device)
    params = [p for p in module.parameters() if p.requires_grad]
    seqpar = bool(cfg.get("seqpar")) and world > 1
    B, T = cfg["B"], cfg["T"]
    shard = None
    if seqpar:
        # every rank holds a contiguous T / world slice of the same sequences
        from thetascan_b200.seqpar import nccl_shard
        if T % world:
            raise SystemExit(f"T={T} does not split into {world} shards")
        shard = nccl_shard()
        gen = torch.Generator(device="cpu").manual_seed(1000)
        L = T // world
        x_host = torch.randn(B, T, cfg["D"], generator=gen)[:, rank * L:(rank + 1) * L]
        x_host = x_host.to(torch.bfloat16).contiguous().pin_memory()
        T = L
    else:
        gen = torch.Generator(device="cpu").manual_seed(1000 + rank)
        xdt = torch.float32 if cfg.get("dtype") == "f32" else torch.bfloat16
        x_host = torch.randn(B, T, cfg["D"], generator=gen).to(xdt).pin_memory()
    x = x_host.to(device)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)

    def step(inp):
        for p in params:
            p.grad = None
        y = module(inp, shard)
        loss = y.float().square().mean()
        loss.backward()
        if world > 1:
            flat = torch.cat([p.grad.reshape(-1) for p in params])
            dist.all_reduce(flat)
            flat.div_(world)
            offset = 0
            for p in params:
                n = p.numel()
                p.grad.copy_(flat[offset:offset + n].view_as(p.grad))
                offset += n
        return loss

    lib = _lib.load()
    timer = PhaseTimer(lib)
    timer.install()
    for _ in range(args.warmup):
        step(x)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches0 = lib.ts_b200_launch_count()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(device_bus_id(local)) as clocks:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        wall0 = time.perf_counter()
        # The timed region is the whole sequence of K steps on each rank (one
        # event pair; the L2 flush between steps, a 256 MB fill of ~0.05 ms,
        # is inside it), so that skew between ranks counts once rather than
        # inside every step; per-step events are kept for the spread.
        region0, region1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        region0.record()
        for i in range(args.steps):
            flush.fill_(float(i))  # evict L2 (256 MB > 126 MB) between timed steps
            starts[i].record()
            step(x)
            ends[i].record()
        region1.record()
        host_ms = (time.perf_counter() - wall0) * 1e3 / args.steps   # enqueue rate (before the drain)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        wall = time.perf_counter() - wall0
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    # the library's own count of the kernels it launched in the timed region
    launches = lib.ts_b200_launch_count() - launches0
    mean_ms = region0.elapsed_time(region1) / args.steps
    if world > 1:
        t = torch.tensor([mean_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        mean_ms = float(t)
    status = _lib.device_status(torch.cuda.current_stream().cuda_stream)

    # Per-entry-point device times (one extra profiled step, not part of the timed region).
    timer.timing = True
    flush.fill_(0.5)
    step(x)
    phase_ms = timer.total_ms()
    timer.timing = False
    timer.uninstall()

    # End-to-end through the public module API, as a training loop runs it:
    # every step's batch is copied from pinned host memory to the device on a
    # copy stream (the copy of step i+1 overlaps step i, as a prefetching input
    # pipeline does; double-buffered device inputs), the step runs
    # forward+backward (and the gradient all-reduce), and its loss is read back
    # into pinned host memory.  The timed region spans the whole sequence of
    # steps, from before the first copy to after the last read-back, with
    # events on the compute stream and a final synchronize.  `serial_ms` is the
    # same step without the overlap (copy, step, read-back, synchronize).
    compute = torch.cuda.current_stream()
    copy_stream = torch.cuda.Stream(device)
    bufs = [torch.empty_like(x), torch.empty_like(x)]
    loss_host = torch.empty(max(args.steps, 3), dtype=torch.float32).pin_memory()

    def e2e_run(n):
        ready = [torch.cuda.Event(), torch.cuda.Event()]
        consumed = [torch.cuda.Event(), torch.cuda.Event()]
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(compute)
        copy_stream.wait_event(start)
        with torch.cuda.stream(copy_stream):
            bufs[0].copy_(x_host, non_blocking=True)
            ready[0].record(copy_stream)
        for i in range(n):
            cur = i % 2
            if i + 1 < n:
                nxt = 1 - cur
                if i >= 1:
                    copy_stream.wait_event(consumed[nxt])   # step i-1 has finished reading it
                with torch.cuda.stream(copy_stream):
                    bufs[nxt].copy_(x_host, non_blocking=True)
                    ready[nxt].record(copy_stream)
            compute.wait_event(ready[cur])
            loss = step(bufs[cur])
            consumed[cur].record(compute)
            loss_host[i].copy_(loss.detach(), non_blocking=True)
        end.record(compute)
        torch.cuda.synchronize()
        return start.elapsed_time(end) / n

    e2e_run(3)                                  # untimed: allocations, pinned staging
    # Two timed repetitions of the K-step sequence; the faster is reported
    # (a host-side stall of the process, e.g. from another tenant of the
    # machine, can stretch one repetition several-fold; both are listed).
    e2e_runs = []
    for rep in range(2):
        flush.fill_(0.25 + rep)
        e2e_runs.append(e2e_run(max(args.steps, 3)))
    if world > 1:
        t = torch.tensor(e2e_runs, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)   # each repetition's slowest rank
        e2e_runs = [float(v) for v in t]
    e2e = min(e2e_runs)
    serial = []
    for i in range(3):
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        bufs[0].copy_(x_host, non_blocking=True)
        loss = step(bufs[0])
        loss_host[0].copy_(loss.detach(), non_blocking=True)
        s1.record()
        torch.cuda.synchronize()
        serial.append(s0.elapsed_time(s1))
    serial_ms = statistics.median(serial)
    if world > 1:
        t = torch.tensor([serial_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        serial_ms = float(t)

    core_flops, mixer_flops, phase_flops = flops_per_token(cfg)
    tokens = B * T * world
    value = tokens / (mean_ms / 1e3)
    peak_sus, peak_burst, peak_hbm, peak_kind = load_peaks()
    # Dominant entry point of ours: algorithmic FLOPs and compulsory bytes per
    # launch; its roofline is the one its arithmetic intensity falls under.
    per_token = {"ts_b200_feature_fwd": phase_flops["feature"], "ts_b200_scan_fwd": phase_flops["scan"],
                 "ts_b200_scan_bwd": 2 * phase_flops["scan"], "ts_b200_feature_bwd": 2 * phase_flops["feature"],
                 "ts_b200_kread_fwd": 0, "ts_b200_kread_bwd": 0}
    dominant = max(phase_ms, key=phase_ms.get)
    launch_s = phase_ms[dominant] / 1e3
    flops_launch = per_token[dominant] * B * T
    bytes_launch = bytes_per_token(cfg)[dominant] * B * T
    ridge = peak_sus * 1e12 / (peak_hbm * 1e9)
    traffic, traffic_source = measured_traffic(dominant, B * T) if args.config in ("c2", "c2b2") else (None, None)
    if cfg.get("dtype") == "f32":
        # float32 scan kernels: f32 FMAs on the CUDA cores (no tensor cores)
        fma_peak = 148 * 128 * 2 * 1.965e9 / 1e12
        achieved = flops_launch / launch_s / 1e12
        roofline = {"bound": "fp32 cuda cores", "kernel": dominant, "achieved": achieved, "peak": fma_peak,
                    "unit": "TFLOP/s", "frac": achieved / fma_peak, "traffic": None,
                    "flops_per_launch": flops_launch,
                    "peak_source": "nominal: 148 SMs x 128 f32 lanes x 2 x 1.965 GHz"}
    elif flops_launch / max(bytes_launch, 1) < ridge:
        achieved = bytes_launch / launch_s / 1e9
        roofline = {"bound": "hbm", "kernel": dominant, "achieved": achieved, "peak": peak_hbm, "unit": "GB/s",
                    "frac": achieved / peak_hbm, "traffic": traffic, "traffic_source": traffic_source,
                    "bytes_per_launch": bytes_launch,
                    "flops_per_launch": flops_launch, "tflops": flops_launch / launch_s / 1e12,
                    "peak_source": f"{peak_kind} hbm_gbs"}
    else:
        achieved = flops_launch / launch_s / 1e12
        roofline = {"bound": "tensor", "kernel": dominant, "achieved": achieved, "peak": peak_sus,
                    "unit": "TFLOP/s", "frac": achieved / peak_sus, "traffic": traffic,
                    "traffic_source": traffic_source,
                    "bytes_per_launch": bytes_launch, "flops_per_launch": flops_launch,
                    "peak_source": f"{peak_kind} bf16_tflops_sustained"}
    # Per GPU: `value` is the whole job's tokens/s, the peak one GPU's.
    mixer_tflops = mixer_flops * value / world / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": mean_ms, "higher_is_better": True,
        "scaling": "strong" if seqpar else "weak",
        "vs_baseline": None, "dtype": "f32" if cfg.get("dtype") == "f32" else "bf16",
        "data": "synthetic x ~ N(0,1), seeded random-init weights",
        "config": {"workload": WORKLOADS.get(args.config, f"{args.config}: {cfg}"),
                   "model": "ThetaScan-Kernel mixer", "global_batch": B if seqpar else B * world,
                   "seq_len": T * world if seqpar else T,
                   "d_model": cfg["D"], "heads": cfg["H"],
                   "parallelism": f"sp{world}" if seqpar else (f"dp{world}" if world > 1 else "single"),
                   "l2": "256 MB buffer written before every timed step"},
        "roofline": roofline,
        "mixer_roofline": {"achieved": mixer_tflops, "peak": peak_sus, "unit": "TFLOP/s", "per": "gpu",
                           "frac": mixer_tflops / peak_sus, "flop_per_token": mixer_flops,
                           "core_flop_per_token": core_flops},
        "phase_ms": {k.replace("ts_b200_", ""): round(v, 4) for k, v in phase_ms.items()},
        "e2e": {"value": tokens / (e2e / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": x_host.numel() * x_host.element_size(), "d2h_bytes_per_step": 4,
                "ms_per_step": e2e, "mode": "pipelined input copies (copy stream, double buffer)",
                "repetitions_ms_per_step": e2e_runs,
                "serial_value": tokens / (serial_ms / 1e3), "serial_ms_per_step": serial_ms},
        "gpu_launches": launches,
        "host_enqueue_ms_per_step": host_ms,
        "step_ms_spread": [min(step_ms), max(step_ms)],
        "clocks": clocks.summary(),
        "wall_s": wall,
        "device_status": status,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.config in ("c1", "c2"):
        # the reference's own CPU code on a bounded sample (c1: its chunk
        # backend on the whole config-1 workload; c2: its cumsum backend, the
        # baseline's CPU arm, on one 1024-token sequence)
        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        view_set, T_cpu, reps = ("bank", T, 3) if args.config == "c1" else ("sum", args.ref_tokens, 1)
        runs = [cpu_reference_step(cfg, T_cpu, view_set) for _ in range(reps)]
        secs = statistics.median(t for t, _ in runs)
        line["cpu_baseline"] = {"value": T_cpu / secs, "unit": "tokens/s", "cores": threads, "kind": runs[0][1],
                                "sample": _reference_sample(runs[0][1], view_set, T_cpu, reps)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_lm(args, cfg):
    """Config 5: whole training steps (forward, backward, gradient all-reduce
    across ranks, AdamW) of the hybrid LM on uniform random tokens."""
    from thetascan_b200.lm import HybridLM
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=__import__("datetime").timedelta(seconds=120))
    device = torch.device("cuda", local)
    if cfg["B"] % world:
        raise SystemExit(f"global batch {cfg['B']} does not split over {world} GPUs")
    B, T = cfg["B"] // world, cfg["T"]
    torch.manual_seed(2)
    model = HybridLM(vocab=cfg["vocab"], d_model=cfg["D"], n_layers=cfg["layers"], n_heads=cfg["H"]).to(device)
    params = [p for p in model.parameters() if p.requires_grad]
    n_params = sum(p.numel() for p in params)
    opt = torch.optim.AdamW(params, lr=3e-4, weight_decay=0.0, fused=True)
    gen = torch.Generator().manual_seed(2)
    tokens_all = torch.randint(0, cfg["vocab"], (cfg["B"], T + 1), generator=gen)
    tok_host = tokens_all[rank * B:(rank + 1) * B].contiguous().pin_memory()
    tok = tok_host.to(device)
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)

    def step(inp):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = model.loss(inp)
        loss.backward()
        if world > 1:
            flat = torch.cat([p.grad.reshape(-1) for p in params])
            dist.all_reduce(flat)
            flat.div_(world)
            offset = 0
            for p in params:
                n = p.numel()
                p.grad.copy_(flat[offset:offset + n].view_as(p.grad))
                offset += n
        opt.step()
        opt.zero_grad(set_to_none=True)
        return loss

    for _ in range(args.warmup):
        step(tok)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    with ClockSampler(device_bus_id(local)) as clocks:
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        r0.record()
        for i in range(args.steps):
            flush.fill_(float(i))
            loss = step(tok)
        r1.record()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    mean_ms = r0.elapsed_time(r1) / args.steps
    # end to end: each step's tokens copied from pinned host memory, the loss read back
    loss_host = torch.empty(1, dtype=torch.float32).pin_memory()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    buf = torch.empty_like(tok)
    e0.record()
    for _ in range(args.steps):
        buf.copy_(tok_host, non_blocking=True)
        loss = step(buf)
        loss_host.copy_(loss.detach().float().reshape(1), non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([mean_ms, e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        mean_ms, e2e_ms = float(t[0]), float(t[1])
    tokens = cfg["B"] * T
    value = tokens / (mean_ms / 1e3)
    # model FLOPs per token: 6 N for the dense weights plus the causal
    # attention score/value products of the attention blocks (3 x 2 x 2 x T/2 x d)
    n_attn = cfg["layers"] - 2
    flop_per_token = 6 * n_params + n_attn * 3 * 2 * 2 * (T / 2) * cfg["D"]
    peak_sus, _, _, peak_kind = load_peaks()
    achieved = flop_per_token * value / world / 1e12
    line = {
        "metric": "hybrid LM training step tokens/s (config 5)", "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": mean_ms,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic uniform token ids (seed 2), seeded random-init weights",
        "config": {"workload": WORKLOADS["c5"], "model": f"hybrid LM, {n_params / 1e6:.2f} M parameters",
                   "global_batch": cfg["B"], "seq_len": T, "parallelism": f"dp{world}" if world > 1 else "single",
                   "l2": "256 MB buffer written before every timed step"},
        "roofline": {"bound": "tensor", "kernel": "whole step", "achieved": achieved, "peak": peak_sus,
                     "unit": "TFLOP/s", "frac": achieved / peak_sus, "traffic": None,
                     "flop_per_token": flop_per_token, "peak_source": f"{peak_kind} bf16_tflops_sustained"},
        "loss": float(loss.detach()),
        "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": tok_host.numel() * tok_host.element_size() * world, "d2h_bytes_per_step": 4,
                "ms_per_step": e2e_ms},
        "clocks": clocks.summary(),
        "device_status": _device_status(),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _device_status():
    from thetascan_b200 import _lib
    return _lib.device_status(torch.cuda.current_stream().cuda_stream)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--config", default="c2", choices=sorted(CONFIGS))
    ap.add_argument("--ref-tokens", type=int, default=1024)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        run_reference(args, cfg)
    elif cfg.get("family") == "lm":
        run_lm(args, cfg)
    else:
        run_b200(args, cfg)


if __name__ == "__main__":
    main()
