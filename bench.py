"""Benchmark of the B200 TurboAdam optimizer step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config llama3-8b|gpt2-block|gpt2-124m|flat-vonly] [--v-bits B]

Prints one JSON line (rank 0). Metric: parameters updated per second per
optimizer step (whole job, all ranks), plus achieved HBM GB/s of the
dominant kernel against the measured B200 copy bandwidth.

Workload (default): the Llama-3-8B parameter set
(8,030,261,248 fp32 params, 291 tensors), random init N(0, 0.02), seeded
N(0, 1e-4) gradients, 4-bit v + CoState, lr 6e-4, wd 0.01. Gradients are
generated once on the device and reused every step (the step does not read
them differently). When a workload's bytes exceed 4x the 126 MB L2 nothing
is flushed between steps; a smaller one (config 1) gets a 512 MB buffer
written between steps and is timed per step. At N > 1 GPUs whole tensors are
assigned to ranks by longest-processing-time (no tensor spans ranks, so the
step has no collective); the total parameter set is fixed, i.e. strong
scaling. Rank 0 also reports every rank's phase times.

The GPT-2 configs follow BASELINE.json: LayerNorm weights 1 and biases 0;
config 2's gradients are N(0, sigma_t) with one sigma_t per tensor drawn
log-uniform in [1e-5, 1e-2] and 5 % of the wte rows zero.

At N = 1 rank 0 also times the reference's own GPU step (its Triton kernels,
from the unmodified install in baseline/_ref) and ours on the same sample
of the workload (``reference_gpu``), and the reference algorithm's CPU
restatement on all host threads and on one (``cpu_baseline``).

--impl reference times the reference algorithm's CPU restatement (oracle/,
C + OpenMP, all host threads) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "params updated/sec per optimizer step"
L2_BYTES = 126 * 1000 * 1000  # B200 L2
UNIT = "params/s"


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------

def llama3_8b_shapes():
    d, kv, ffn, vocab, L = 4096, 1024, 14336, 128256, 32
    shapes = [("embed", (vocab, d))]
    for i in range(L):
        shapes += [(f"l{i}.q", (d, d)), (f"l{i}.k", (kv, d)), (f"l{i}.v", (kv, d)),
                   (f"l{i}.o", (d, d)), (f"l{i}.gate", (ffn, d)), (f"l{i}.up", (ffn, d)),
                   (f"l{i}.down", (d, ffn)), (f"l{i}.ln1", (d,)), (f"l{i}.ln2", (d,))]
    shapes += [("norm", (d,)), ("lm_head", (vocab, d))]
    return shapes


def gpt2_block_shapes(prefix=""):
    return [(prefix + "ln_1.w", (768,)), (prefix + "ln_1.b", (768,)),
            (prefix + "c_attn.w", (768, 2304)), (prefix + "c_attn.b", (2304,)),
            (prefix + "attn.c_proj.w", (768, 768)), (prefix + "attn.c_proj.b", (768,)),
            (prefix + "ln_2.w", (768,)), (prefix + "ln_2.b", (768,)),
            (prefix + "c_fc.w", (768, 3072)), (prefix + "c_fc.b", (3072,)),
            (prefix + "mlp.c_proj.w", (3072, 768)), (prefix + "mlp.c_proj.b", (768,))]


def gpt2_124m_shapes():
    s = [("wte", (50257, 768)), ("wpe", (1024, 768))]
    for i in range(12):
        s += gpt2_block_shapes(f"h{i}.")
    s += [("ln_f.w", (768,)), ("ln_f.b", (768,))]
    return s


def llama3_70b_shapes():
    d, kv, ffn, vocab, L = 8192, 1024, 28672, 128256, 80
    shapes = [("embed", (vocab, d))]
    for i in range(L):
        shapes += [(f"l{i}.q", (d, d)), (f"l{i}.k", (kv, d)), (f"l{i}.v", (kv, d)),
                   (f"l{i}.o", (d, d)), (f"l{i}.gate", (ffn, d)), (f"l{i}.up", (ffn, d)),
                   (f"l{i}.down", (d, ffn)), (f"l{i}.ln1", (d,)), (f"l{i}.ln2", (d,))]
    shapes += [("norm", (d,)), ("lm_head", (vocab, d))]
    return shapes


CONFIGS = {
    "llama3-8b": dict(shapes=llama3_8b_shapes, kw=dict(lr=6e-4, weight_decay=0.01, v_bits=4),
                      grad_std=1e-4, dtype="fp32"),
    # bf16 params and grads, 3-bit v + CoState, ZeRO-1 at 4 and 8 GPUs
    "llama3-70b": dict(shapes=llama3_70b_shapes, kw=dict(lr=6e-4, weight_decay=0.01, v_bits=3),
                       grad_std=1e-4, dtype="bf16", partition="zero1"),
    # LayerNorm weights 1, biases 0, N(0, 1e-3) gradients
    "gpt2-block": dict(shapes=gpt2_block_shapes, kw=dict(lr=6e-4, weight_decay=0.01, v_bits=4),
                       grad_std=1e-3, dtype="fp32", init="gpt2"),
    # per-tensor sigma log-uniform in [1e-5, 1e-2], 5 % zero wte rows
    "gpt2-124m": dict(shapes=gpt2_124m_shapes, kw=dict(lr=6e-4, weight_decay=0.01, v_bits=4),
                      grad_std=1e-3, dtype="fp32", init="gpt2", grad_dist="gpt2_c2"),
    # Student-t (nu = 3) gradients scaled by 1e-3
    "flat-vonly": dict(shapes=lambda: [("flat", (2 ** 30 + 37,))],
                       kw=dict(lr=1e-3, compress_m=False, v_bits=4), grad_std=1e-3,
                       dtype="fp32", grad_dist="student_t3"),
}


def student_t3_(out, scale, gen, chunk=1 << 26):
    """out <- scale * Z / sqrt(chi2_3 / 3) (Student-t, 3 degrees of freedom),
    generated on the device in chunks."""
    import torch

    flat = out.view(-1)
    for lo in range(0, flat.numel(), chunk):
        n = min(chunk, flat.numel() - lo)
        z = torch.randn(4, n, device=out.device, generator=gen)
        chi = (z[1] * z[1] + z[2] * z[2] + z[3] * z[3]) / 3.0
        flat[lo:lo + n].copy_(z[0] / chi.sqrt() * scale)
    return out


def init_param_(p, name, cfg, gen):
    """BASELINE init: N(0, 0.02); the GPT-2 configs' LayerNorm weights 1 and
    biases 0."""
    if cfg.get("init") == "gpt2" and name.endswith(".b"):
        return p.zero_()
    if cfg.get("init") == "gpt2" and name.endswith(".w") and "ln_" in name:
        return p.fill_(1.0)
    return p.normal_(0.0, 0.02, generator=gen)


def grad_sigma(cfg, t):
    """Gradient scale of global tensor t (config 2: log-uniform per tensor)."""
    if cfg.get("grad_dist") == "gpt2_c2":
        return float(10.0 ** np.random.default_rng(5000 + t).uniform(-5.0, -2.0))
    return cfg["grad_std"]


def make_grad(p, name, t, cfg, gen, row0=0):
    """Seeded synthetic gradient of (a shard starting at flat element row0 of)
    global tensor t, in p's shape and dtype."""
    import torch

    sig = grad_sigma(cfg, t)
    if cfg.get("grad_dist") == "student_t3":
        return student_t3_(torch.empty_like(p), sig, gen)
    g = torch.empty_like(p).normal_(0.0, sig, generator=gen)
    if cfg.get("grad_dist") == "gpt2_c2" and name == "wte":
        # 5 % of the embedding rows (768 = 6 blocks each) get zero gradient
        rows = g.view(-1, 768)
        mask = torch.from_numpy(np.random.default_rng(6000).random(50257) < 0.05)
        r0 = row0 // 768
        rows[mask[r0:r0 + rows.shape[0]].to(g.device)] = 0.0
    return g


def numel(shape):
    n = 1
    for s in shape:
        n *= s
    return n


def lpt_assign(shapes, world):
    from turboadam_b200.sharding import lpt_owners

    return lpt_owners([numel(s) for _, s in shapes], world)


def kind_of(n, kw, n_policy=None):
    n_policy = n if n_policy is None else n_policy  # shards decide by the whole tensor
    costate = kw.get("compress_m", True) and n_policy >= kw.get("min_m_compress_elements", 4096)
    oneq = kw.get("compress_v", True)
    return costate, oneq


def pass1_bytes(n, kw, psize=4, n_policy=None):
    """Algorithmic HBM bytes of pass 1 for one tensor: read+write p, read g,
    read the old m state, read+write the v state (u8 layout)."""
    costate, oneq = kind_of(n, kw, n_policy)
    B = (n + 127) // 128
    b = 2 * psize * n + psize * n
    b += (n + 7) // 8 + 7 * B if costate else 8 * n
    b += 2 * 128 * B + 8 * B if oneq else 8 * n
    return b


def step_bytes(n, kw, psize=4, n_policy=None):
    """Single-touch algorithmic bytes of the whole step (figures:
    14.42 B/param for 4-bit + CoState fp32, 22.06 v-only fp32, 8.42 3-bit +
    CoState bf16)."""
    costate, oneq = kind_of(n, kw, n_policy)
    B = (n + 127) // 128
    b = 3 * psize * n
    b += 2 * ((n + 7) // 8) + 14 * B if costate else 8 * n
    b += 2 * 128 * B + 8 * B if oneq else 8 * n
    return b


# ---------------------------------------------------------------------------
# clocks sampling (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------

class Clocks:
    """SM clock and clock-event (throttle) reasons of this rank's GPU during
    the timed region. NVML is read from a thread every 10 ms and once more
    when the region ends (the GPU has just finished its last step then), so
    even a region of a few milliseconds has samples; without NVML bindings
    `nvidia-smi -lms 200` runs alongside (a region shorter than its start-up
    may then have none). Reading clocks changes no setting."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    # NVML clocks-event reason bits (nvml.h nvmlClocksEventReason*)
    REASONS = (("sw_power_cap", 0x4), ("hw_slowdown", 0x8), ("sw_thermal_slowdown", 0x20),
               ("hw_thermal_slowdown", 0x40), ("hw_power_brake_slowdown", 0x80))

    def __init__(self, index, device=None):
        self.index = index
        self.device = device
        self.proc = None
        self.path = None
        self.nvml = None
        self.samples = []
        self.thread = None
        self.halt = None

    def _nvml_handle(self):
        import pynvml

        pynvml.nvmlInit()
        if self.device is not None:
            try:
                import torch

                pr = torch.cuda.get_device_properties(self.device)
                bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
                return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            except Exception:
                pass
        return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def _read(self):
        nv, h = self.nvml
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        self.samples.append((sm, mx, rs))

    def start(self):
        try:
            import threading

            self.nvml = self._nvml_handle()
            self.halt = threading.Event()

            def poll():
                while not self.halt.wait(0.01):
                    try:
                        self._read()
                    except Exception:
                        return

            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            return
        except Exception:
            self.nvml = None
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.nvml is not None:
            self.halt.set()
            self.thread.join(timeout=5)
            try:
                self._read()
            except Exception:
                pass
            reasons = sorted({nm for _, _, rs in self.samples for nm, bit in self.REASONS
                              if rs & bit})
            return {"sm_mhz": statistics.median(sm for sm, _, _ in self.samples),
                    "sm_max_mhz": max(mx for _, mx, _ in self.samples),
                    "reasons": reasons, "samples": len(self.samples), "source": "nvml"}
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        os.unlink(self.path)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx),
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi"}


# ---------------------------------------------------------------------------
# CPU baseline: the reference algorithm restated in C (oracle/), all threads
# ---------------------------------------------------------------------------

def _cpu_pick(cfg_name, shapes):
    """Bounded CPU sample: the attention tensors + norms of layer 0 for
    Llama-3-8B (42M params), a 2^24+37 slice for the flat tensor, else all."""
    if cfg_name == "llama3-8b":
        return [s for s in shapes if s[0] in ("l0.q", "l0.k", "l0.v", "l0.o", "l0.ln1", "l0.ln2")]
    if cfg_name == "flat-vonly":
        return [("flat_sample", (2 ** 24 + 37,))]
    return shapes


def np_sample_tensors(cfg_name, rng):
    """The CPU sample's parameters and gradients (numpy), initialised as the
    GPU workload is (BASELINE init and gradient model)."""
    from oracle import oracle as O

    cfg = CONFIGS[cfg_name]
    shapes = cfg["shapes"]()
    pick = _cpu_pick(cfg_name, shapes)
    index = {name: t for t, (name, _) in enumerate(shapes)}
    params = []
    for name, shp in pick:
        n = numel(shp)
        if cfg.get("init") == "gpt2" and name.endswith(".b"):
            x = np.zeros(n, np.float32)
        elif cfg.get("init") == "gpt2" and name.endswith(".w") and "ln_" in name:
            x = np.ones(n, np.float32)
        else:
            x = rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)
        p = O.OracleParam(x)
        g = rng.standard_normal(n, dtype=np.float32) * np.float32(
            grad_sigma(cfg, index.get(name, 0)))
        if cfg.get("grad_dist") == "gpt2_c2" and name == "wte":
            g.reshape(-1, 768)[np.random.default_rng(6000).random(50257) < 0.05] = 0.0
        p.grad = g
        params.append(p)
    return pick, params


def cpu_cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def cpu_sample(cfg_name, target_s=12.0):
    """Times the CPU restatement of the step on a bounded sample of the
    workload (whole tensors, in workload order) on all host threads, and
    then on one thread."""
    import torch

    from oracle import oracle as O

    O.build()
    threads = len(os.sched_getaffinity(0))
    cfg = CONFIGS[cfg_name]
    kw = cfg["kw"]
    pick, params = np_sample_tensors(cfg_name, np.random.default_rng(0))
    n_total = sum(p.n for p in params)

    def timed(nthreads, budget):
        O.set_threads(nthreads)
        opt = O.OracleTurboAdam([O.OracleTurboAdam.make_group(params, **kw)])
        times = []
        t_all = time.perf_counter()
        while True:
            t0 = time.perf_counter()
            opt.step(uniforms=lambda i, st, npad: O.sr_uniforms(params[i].n, i, st, 1))
            times.append(time.perf_counter() - t0)
            if time.perf_counter() - t_all > budget or len(times) >= 50:
                break
        return statistics.median(times), len(times)

    best, nsteps = timed(threads, target_s)
    best1, nsteps1 = timed(1, target_s / 2)
    O.set_threads(threads)
    names = ",".join(n for n, _ in pick)
    return {
        "value": n_total / best,
        "unit": UNIT,
        "cores": threads,
        "kind": "port",
        "sample": f"{len(pick)} tensors ({n_total} params: {names[:80]}"
                  f"{'...' if len(names) > 80 else ''}), {nsteps} steps, median step "
                  f"{best * 1e3:.1f} ms, SR uniforms from the same Philox stream",
        "single_thread": {"value": n_total / best1, "cores": 1, "steps": nsteps1,
                          "ms_per_step": best1 * 1e3},
        "cpu_model": cpu_cpu_model(),
        "host_threads_available": threads,
        "torch": torch.__version__,
    }


def run_reference(args, rank, world):
    if rank != 0:
        return
    cfg = CONFIGS[args.config]
    from oracle import oracle as O

    O.build()
    O.set_threads(len(os.sched_getaffinity(0)))  # all host cores (torchrun sets 1)
    pick, params = np_sample_tensors(args.config, np.random.default_rng(0))
    opt = O.OracleTurboAdam([O.OracleTurboAdam.make_group(params, **cfg["kw"])])
    ufn = lambda i, st, npad: O.sr_uniforms(params[i].n, i, st, 1)  # noqa: E731
    for _ in range(args.warmup):
        opt.step(uniforms=ufn)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        opt.step(uniforms=ufn)
    dt = (time.perf_counter() - t0) / args.steps
    n_total = sum(p.n for p in params)
    val = n_total / dt
    sample = f"{len(pick)} tensors of {args.config} ({n_total} params) per step"
    out = {
        "impl": "reference", "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": args.config, "sample_params": n_total},
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": O.threads(), "kind": "port",
                         "sample": sample, "cpu_model": cpu_cpu_model()},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(out), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------

def _gpu_ref_pick(cfg_name, shapes):
    """Sample of the workload for the reference's GPU step: one transformer
    layer of the Llama configs (its Python loop is per tensor; a layer has
    every tensor kind), a 2^26 + 37 slice of the flat tensor, else all."""
    if cfg_name in ("llama3-8b", "llama3-70b"):
        return [(t, s) for t, s in enumerate(shapes) if s[0].startswith("l0.")]
    if cfg_name == "flat-vonly":
        return [(0, ("flat", (2 ** 26 + 37,)))]
    return list(enumerate(shapes))


def reference_gpu(cfg_name, kw, dev, steps=3, warmup=2):
    """The reference's own optimizer step on this GPU -- TurboAdam.step() of
    the unmodified package installed in baseline/_ref, whose CUDA path runs
    its Triton kernels (triton_kernels.py) -- and ours, timed on the same
    sample tensors with CUDA events around each step() call."""
    import torch

    from turboadam_b200 import TurboAdam

    ref_dir = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "turboadam")):
        return {"unavailable": "the reference is not installed in baseline/_ref"}
    sys.path.insert(0, ref_dir)
    try:
        import turboadam as ref
        from turboadam import optimizer as ref_optimizer
    except Exception as e:  # pragma: no cover
        return {"unavailable": f"import of the reference failed: {e!r}"}
    finally:
        sys.path.remove(ref_dir)
    if not getattr(ref_optimizer, "_HAS_TRITON", False):
        return {"unavailable": "the reference's Triton kernels did not import"}
    cfg = CONFIGS[cfg_name]
    shapes = cfg["shapes"]()
    pick = _gpu_ref_pick(cfg_name, shapes)
    pdtype = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float32
    gen = torch.Generator(device=dev)

    def tensors():
        ps = []
        for t, (name, shp) in pick:
            gen.manual_seed(1234 + 7919 * t)
            p = torch.nn.Parameter(init_param_(torch.empty(shp, dtype=pdtype, device=dev), name,
                                               cfg, gen))
            p.grad = make_grad(p, name, t, cfg, gen)
            ps.append(p)
        return ps

    def timed(opt):
        for _ in range(warmup):
            opt.step()
        torch.cuda.synchronize(dev)
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
        evs[0].record()
        for k in range(steps):
            opt.step()
            evs[k + 1].record()
        torch.cuda.synchronize(dev)
        return [evs[k].elapsed_time(evs[k + 1]) for k in range(steps)]

    n = sum(numel(s) for _, (_, s) in pick)
    try:
        ps = tensors()
        ref_ms = timed(ref.TurboAdam(ps, betas=(0.9, 0.999), **kw))
        del ps
        torch.cuda.empty_cache()
        ps = tensors()
        our_ms = timed(TurboAdam(ps, betas=(0.9, 0.999), seed=2024, **kw))
        del ps
        torch.cuda.empty_cache()
    except Exception as e:
        return {"unavailable": f"the reference's GPU step failed: {e!r}"[:300]}
    rm, om = statistics.median(ref_ms), statistics.median(our_ms)
    return {
        "value": n / (rm / 1e3), "unit": UNIT, "ms_per_step": rm,
        "ours_ms_per_step": om, "ours_value": n / (om / 1e3), "speedup": rm / om,
        "sample": f"{len(pick)} tensors of {cfg_name} ({n} params: "
                  f"{','.join(s[0] for _, s in pick)[:80]}), {warmup} warm-up + {steps} timed "
                  "steps each, CUDA events around step(), median",
        "path": "reference TurboAdam.step() on CUDA tensors from baseline/_ref (unmodified): "
                "Triton fused_v_update + CoState codec, torch ops for the rest",
    }


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic(config):
    """Per-param DRAM bytes of pass 1 from the committed ncu summary of the
    same kernel kind (fp32 CoState + 4-bit 1Q: a GPT-2 124M capture; bf16
    CoState + 3-bit: one Llama-3-70B layer). The traffic per element does not
    depend on the tensor count, so it scales to a full launch by the elements
    processed; a config whose kernel kind has no capture gets None."""
    name = {"llama3-8b": "k_pass1_gpt2-124m.txt", "gpt2-124m": "k_pass1_gpt2-124m.txt",
            "gpt2-block": "k_pass1_gpt2-124m.txt",
            "llama3-70b": "k_pass1_llama3-70b-layer.txt"}.get(config)
    p = os.path.join(ROOT, "profiles", name) if name else None
    if p is None or not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("dram_bytes_per_param"):
            try:
                return float(line.split("=")[1].split()[0])
            except Exception:
                return None
    return None


def run_ours(args, rank, world, local_rank):
    import torch

    from turboadam_b200 import TurboAdam

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    cfg = CONFIGS[args.config]
    shapes = cfg["shapes"]()
    if args.layers:  # a labelled subset: the first L transformer layers, no embedding / head
        shapes = [s for s in shapes if any(s[0].startswith(f"l{i}.") for i in range(args.layers))]
    kw = dict(cfg["kw"])
    if args.v_bits:
        kw["v_bits"] = args.v_bits
    part = args.partition if args.partition != "auto" else cfg.get("partition", "tensor")
    if args.layers and world == 1:
        part = "tensor"
    pdtype = torch.bfloat16 if cfg["dtype"] == "bf16" else torch.float32
    psize = 2 if cfg["dtype"] == "bf16" else 4
    # local tensors: (shape, global tensor index, shard (block_offset, global_numel) or None)
    if part == "zero1":
        from turboadam_b200.sharding import zero1_partition, zero1_spanning

        parts = zero1_partition([numel(s) for _, s in shapes], world)
        local = [((e1 - e0,), t, (boff, gn)) for t, e0, e1, boff, gn in parts[rank]]
        spanning = zero1_spanning(parts)
        # the gpt2 init and the wte zero rows need the tensor names; a shard
        # of wte starts at whole rows only if it starts at element 0
        row0 = {t: e0 for t, e0, _, _, _ in parts[rank]}
    else:
        owner = lpt_assign(shapes, world)
        local = [(shapes[i][1], i, None) for i in range(len(shapes)) if owner[i] == rank]
        spanning = None
        row0 = {}
    mine = [(numel(shp), sh[1] if sh else numel(shp)) for shp, _, sh in local]  # (n, n_policy)
    total_params = sum(numel(s) for _, s in shapes)
    my_params = sum(n for n, _ in mine)
    gen = torch.Generator(device=dev)
    params = []
    for shp, t, sh in local:  # data keyed by the global tensor (and shard) index
        gen.manual_seed(1234 + 7919 * t + (sh[0] // 4096 if sh else 0))
        name = shapes[t][0]
        p = init_param_(torch.empty(shp, dtype=pdtype, device=dev), name, cfg, gen)
        p = torch.nn.Parameter(p)
        if name == "wte" and row0.get(t, 0) % 768:
            raise ValueError("a wte shard must start at a whole row")
        p.grad = make_grad(p, name, t, cfg, gen, row0.get(t, 0))
        params.append(p)
    opt = TurboAdam(params, betas=(0.9, 0.999), seed=2024, tensor_ids=[t for _, t, _ in local],
                    shards=[sh for _, _, sh in local] if part == "zero1" else None,
                    spanning=spanning, **kw)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            import torch.distributed as dist

            dist.barrier()

    for _ in range(max(args.warmup, 0)):
        opt.step()
    torch.cuda.synchronize(dev)

    # per-step phase events (pass 1, alpha, pass 2, select+labels)
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
    for row in evs:
        for e in row:
            e.record(stream)
    torch.cuda.synchronize(dev)
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    clocks = Clocks(local_rank, dev)
    # a working set that L2 could hold between steps is timed per step, with
    # a 512 MB buffer written between steps (outside the step's events)
    ws_bytes = sum(step_bytes(n, kw, psize, npol) for n, npol in mine)
    flush = ws_bytes < 4 * L2_BYTES
    fbuf = torch.empty(512 << 20, dtype=torch.uint8, device=dev) if flush else None
    barrier()
    torch.cuda.synchronize(dev)
    clocks.start()
    t_start.record(stream)
    for k in range(args.steps):
        if flush:
            fbuf.fill_(k & 0xFF)
        opt._phase_events = evs[k]
        opt.step()
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    barrier()
    opt._phase_events = None
    if flush:
        ms = sum(row[0].elapsed_time(row[4]) for row in evs) / args.steps
    else:
        ms = t_start.elapsed_time(t_end) / args.steps
    phase = np.zeros(4)
    for row in evs:
        for i in range(4):
            phase[i] += row[i].elapsed_time(row[i + 1])
    phase /= args.steps
    del fbuf
    status = opt.read_status()
    per_rank = None
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
        mine_t = torch.tensor([ms, *phase.tolist(), float(my_params)], dtype=torch.float64,
                              device=dev)
        allr = [torch.empty_like(mine_t) for _ in range(world)]
        dist.all_gather(allr, mine_t)
        per_rank = [{"rank": r, "ms_per_step": float(x[0]), "params": int(x[5]),
                     "phase_ms": {"pass1": float(x[1]), "alpha": float(x[2]),
                                  "pass2": float(x[3]), "select_labels": float(x[4])}}
                    for r, x in enumerate(allr)]
    else:
        ms_max = ms

    # ---- end to end through the public API with host buffers: every step
    # copies its gradients host -> device and the updated parameters device ->
    # host. Gradients are double-buffered so the next step's upload (h2d
    # stream) runs while this step's parameters download (d2h stream): the
    # two PCIe directions overlap; the step itself waits for its gradients,
    # and the next step waits for the download of the parameters it updates.
    e2e = None
    if args.e2e_steps > 0:
        largest = max(p.numel() for p in params)
        h_in = torch.empty(largest, dtype=pdtype, pin_memory=True)
        h_in.normal_(0.0, cfg["grad_std"])
        h_out = torch.empty(largest, dtype=pdtype, pin_memory=True)
        gbuf = [[p.grad for p in params], [torch.empty_like(p) for p in params]]
        s_h2d, s_d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        h2d = sum(p.numel() * psize for p in params)

        def upload(k):
            with torch.cuda.stream(s_h2d):
                for g, p in zip(gbuf[k % 2], params):
                    g.view(-1).copy_(h_in[: p.numel()], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(s_h2d)
            return ev

        barrier()
        torch.cuda.synchronize(dev)
        e0.record(stream)
        s_h2d.wait_stream(stream)
        s_d2h.wait_stream(stream)
        ready = upload(0)
        down = None
        for k in range(args.e2e_steps):
            stream.wait_event(ready)
            if down is not None:
                stream.wait_event(down)  # the step rewrites the parameters being read
            for g, p in zip(gbuf[k % 2], params):
                p.grad = g
            opt.step()
            stepped = torch.cuda.Event()
            stepped.record(stream)
            if k + 1 < args.e2e_steps:
                s_h2d.wait_event(stepped)  # the other buffer was read by step k - 1
                ready = upload(k + 1)
            with torch.cuda.stream(s_d2h):
                s_d2h.wait_event(stepped)
                for p in params:  # one landing buffer (bandwidth, not retention)
                    h_out[: p.numel()].copy_(p.detach().view(-1), non_blocking=True)
                down = torch.cuda.Event()
                down.record(s_d2h)
        stream.wait_event(down)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        for p, g in zip(params, gbuf[0]):
            p.grad = g
        del gbuf
        e_ms = e0.elapsed_time(e1) / args.e2e_steps
        if world > 1:
            import torch.distributed as dist

            t = torch.tensor([e_ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            e_ms = float(t.item())
        e2e = {"value": total_params / (e_ms / 1e3), "unit": UNIT, "h2d_bytes_per_step": h2d,
               "d2h_bytes_per_step": h2d, "ms_per_step": e_ms,
               "path": "grads H2D from pinned host memory (double-buffered, overlapping the "
                       "previous step's D2H), TurboAdam.step(), updated params D2H to pinned "
                       "host memory, per tensor"}

    if rank != 0:
        return
    peak, peak_kind = measured_peak()
    p1_bytes = sum(pass1_bytes(n, kw, psize, npol) for n, npol in mine)
    st_bytes = sum(step_bytes(n, kw, psize, npol) for n, npol in mine)
    achieved = p1_bytes / (phase[0] * 1e-3) / 1e9
    tpp = profiled_traffic(args.config)
    n_costate = sum(1 for n, npol in mine if kind_of(n, kw, npol)[0])
    kinds = {kind_of(n, kw, npol) for n, npol in mine}
    launches_per_step = len(kinds) + (1 + 1 + 4 if n_costate else 0)
    out = {
        "metric": METRIC,
        "value": total_params / (ms_max / 1e3),
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_max,
        "higher_is_better": True,
        "scaling": "strong" if world > 1 else "strong",
        "vs_baseline": None,
        "dtype": "bf16" if psize == 2 else "f32",
        "data": ("synthetic: random-init params N(0,0.02), seeded %s grads generated on "
                 "device once and reused each step"
                 % ("Student-t(3) x %g" % cfg["grad_std"] if cfg.get("grad_dist") == "student_t3"
                    else "N(0,%g)" % cfg["grad_std"])),
        "config": {"workload": args.config + (f"[first {args.layers} layers]" if args.layers
                                              else ""),
                   "params": total_params, "tensors": len(shapes),
                   "v_bits": kw["v_bits"], "costate": kw.get("compress_m", True),
                   "parallelism": (f"ZeRO-1 flat partition over {world} GPU(s); " + (
                                       f"{len(spanning)} tensor(s) split at 4096-block "
                                       "boundaries, 4 all-reduces per step (alpha chunk sums, 3 "
                                       "histogram rounds)" if spanning else
                                       "every cut falls on a tensor boundary: no tensor is "
                                       "split, no collective") if part == "zero1" else
                                   f"by-tensor LPT over {world} GPU(s), no collective"),
                   "l2": (f"{ws_bytes / 1e6:.0f} MB per rank per step < 4 x 126 MB L2: a 512 MB "
                          "buffer is written between steps, each step timed by its own events"
                          if flush else f"{ws_bytes / 1e9:.1f} GB per rank per step exceed the "
                          "126 MB L2; no flush")},
        "roofline": {
            "bound": "hbm",
            "kernel": "k_pass1 (weight decay + m + 1Q v + AdamW, one HBM pass)",
            "achieved": achieved,
            "peak": peak,
            "unit": "GB/s",
            "frac": achieved / peak,
            "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)",
            "algorithmic_bytes_per_launch": p1_bytes,
            "ms_per_launch": phase[0],
            "traffic": (tpp * my_params) if tpp else None,
        },
        "step_roofline": {
            "bytes_per_param_single_touch": st_bytes / my_params,
            "achieved": st_bytes / (ms / 1e3) / 1e9,
            "frac": st_bytes / (ms / 1e3) / 1e9 / peak,
            "phase_ms": {"pass1": phase[0], "alpha": phase[1], "pass2": phase[2],
                         "select_labels": phase[3]},
        },
        "gpu_launches": launches_per_step * args.steps,
        "device_status": status,
    }
    if per_rank:
        out["per_rank"] = per_rank
    if clk:
        out["clocks"] = clk
    if e2e:
        out["e2e"] = e2e
    if world == 1 and not args.no_reference_gpu:
        del opt, params
        torch.cuda.empty_cache()
        out["reference_gpu"] = reference_gpu(args.config, kw, dev)
    if world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_sample(args.config)
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="llama3-8b", choices=sorted(CONFIGS))
    ap.add_argument("--v-bits", type=int, default=0)
    ap.add_argument("--partition", default="auto", choices=["auto", "tensor", "zero1"])
    ap.add_argument("--e2e-steps", type=int, default=4)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--layers", type=int, default=0,
                    help="Llama configs: time only the first L transformer layers (a labelled "
                         "subset, e.g. the 70B shape on one GPU)")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip timing the reference's own GPU step (baseline/_ref)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
