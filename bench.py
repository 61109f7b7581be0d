"""Benchmark of the VDN-H3 hybrid block forward on B200 (BASELINE.json metric).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--config 1|3]

One step = one hybrid block forward (QKV, VDA branch, window softmax, gate, out-projection
with the branch delta) of configs[1] of BASELINE.json: 31 latent frames x 836 tokens
(38x22 grid) + 512 text rows, H=40, D=128, hidden 5120, bf16, seeded N(0, 0.02) weights
and N(0, 1) activations (synthetic: no checkpoint or dataset is involved).

Printed JSON line: ``value`` is whole-job TFLOP/s over the algorithmic FLOPs of the block
(allowed attention pairs only) with inputs resident in HBM; ``e2e`` is the same metric
through the public operator (``make_vdn_forward``) with the input copied from pinned host
memory and the output read back every step.  ``roofline`` covers the dominant kernel,
timed with CUDA events on its launch stream inside the timed steps.  ``cpu_baseline`` is
one full block forward of the same weights and input on the host cores (the reference
torch path restated: bf16 GEMMs, fp32 branch), and ``parity_rel_l2`` the relative L2
between its output and the GPU's, over every row.  ``--impl reference`` times that CPU
block forward as its step.

Kernel-only modes for profiling: ``--only attention [--heads n]`` (the window attention kernel
on the config geometry), ``--only quantisers`` (the int8, ConvRot int8 and per-tensor e4m3
activation quantisers on the config's branch rows, against the measured HBM bandwidth),
``--only gemms --precision bf16|int8|fp8 [--rows m]`` (the block's QKV projection GEMM) and
``--only convs`` (the branch's spatial 5x5 and temporal 5-tap convs of the k features).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

PEAK_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
CONFIGS = {
    1: dict(text=512, frames=31, grid=(38, 22), heads=40, dim=128, hidden=5120),
    3: dict(text=512, frames=31, grid=(80, 48), heads=40, dim=128, hidden=5120),
    # the 50-block denoiser stack: DiT blocks (GELU 4x MLP, INT8 projections), CFG batch 2
    4: dict(text=512, frames=31, grid=(38, 22), heads=40, dim=128, hidden=5120, blocks=50, ffn_mult=4,
            activation="gelu", precision="int8", cfg_batch=2, sampler_steps=8),
}


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return dict(PEAK_FALLBACK), "fallback"


def attention_traffic(heads_per_rank: int, heads_total: int):
    """DRAM bytes (read + write) of one window-attention launch, from the committed ncu
    summary of the config-1 geometry (scaled by the head count: every head is a separate
    q/k/v/out slab), or None when the summary is absent."""
    path = os.path.join(ROOT, "profiles", "window_attention_config1_8heads.txt")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch_40_heads:"):
                    return float(line.split(":")[1]) * heads_per_rank / 40.0
    except OSError:
        pass
    return None


class ClockSampler:
    """SM clock and throttle reasons sampled from before the warm-up to after the timed
    region: NVML polled every 5 ms from a thread (nvidia-smi every 50 ms when NVML is not
    importable).  ``mark_start()`` / ``mark_end()`` bracket the timed region on the clock the
    samples are stamped with; ``summary()`` keeps the samples inside it (or, for a region
    shorter than the sampling period, the nearest one on each side).  Read-only: nothing
    here changes a GPU setting."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    NVML_BITS = (0x8, 0x40, 0x20, 0x4)  # the NAMES' bits in NVML's clocks-event-reason mask
    PERIOD_S = 0.005

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.rows: list[tuple[float, float, float, tuple]] = []  # (t, sm_mhz, max_mhz, active names)
        self.t0 = self.t1 = None
        self._stop = False
        self._t = None
        self.source = None

    def start(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            handle = self._nvml_handle(pynvml)
            self.source = "nvml"
            self._t = threading.Thread(target=self._poll_nvml, args=(pynvml, handle), daemon=True)
            self._t.start()
            return self
        except Exception:
            pass
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.source = "nvidia-smi"
            self._t = threading.Thread(target=self._read_smi, daemon=True)
            self._t.start()
        except Exception:
            self.proc = None
        return self

    def _nvml_handle(self, pynvml):
        # the CUDA device's own PCI address, so a remapped CUDA_VISIBLE_DEVICES cannot mislead
        try:
            props = torch.cuda.get_device_properties(self.index)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.index)

    def _poll_nvml(self, pynvml, handle):
        max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(handle, pynvml.NVML_CLOCK_SM))
        while not self._stop:
            try:
                sm = float(pynvml.nvmlDeviceGetClockInfo(handle, pynvml.NVML_CLOCK_SM))
                mask = int(pynvml.nvmlDeviceGetCurrentClocksEventReasons(handle))
                active = tuple(n for n, b in zip(self.NAMES, self.NVML_BITS) if mask & b)
                self.rows.append((time.monotonic(), sm, max_mhz, active))
            except Exception:
                pass
            time.sleep(self.PERIOD_S)

    def _read_smi(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.strip().split(",")]
            if len(parts) < 9:
                continue
            try:
                active = tuple(n for n, v in zip(self.NAMES, parts[5:9]) if v.lower().startswith("active"))
                self.rows.append((time.monotonic(), float(parts[1]), float(parts[2]), active))
            except ValueError:
                continue

    def mark_start(self):
        self.t0 = time.monotonic()

    def mark_end(self):
        self.t1 = time.monotonic()

    def stop(self):
        time.sleep(0.06)  # let the sample after the timed region arrive
        self._stop = True
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self._t is not None:
            self._t.join(timeout=2)

    def summary(self):
        rows = list(self.rows)
        window = "timed region"
        picked = [r for r in rows if self.t0 is not None and self.t0 <= r[0] <= self.t1]
        if not picked and rows and self.t0 is not None:
            before = [r for r in rows if r[0] < self.t0]
            after = [r for r in rows if r[0] > self.t1]
            picked = ([before[-1]] if before else []) + ([after[0]] if after else [])
            window = "nearest samples around a timed region shorter than the sampling period"
        sm = sorted(r[1] for r in picked)
        reasons = sorted({n for r in picked for n in r[3]})
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": picked[-1][2] if picked else None,
                "reasons": reasons, "samples": len(sm), "window": window, "source": self.source}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class ReferenceCPU:
    """The reference's block forward on the host cores: the CPU restatement of its torch path
    (hybrid.py:409-579) at config 1's dtype -- bf16 operands and results for the projections
    and the two attention products (the reference's grouped window backend, window.py:277-313,
    on gathered keys), the branch statistics, factor and scans in fp32 (branch.py:197-243) --
    on every head and every row, with all host threads.  Weights are cast to bf16 once, as
    the reference holds them."""

    def __init__(self, c, weights, x_bf16):
        from oracle import vdn_oracle as vo

        self.vo = vo
        self.c = c
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        qkv, qn, kn, out_w, branch = weights
        br = dict(branch)
        br["to_out_linear.weight"] = br["to_out_linear.weight"].to(torch.bfloat16)
        self.bw = vo.BlockWeights(qkv=qkv.cpu().to(torch.bfloat16), q_norm=qn.cpu(), k_norm=kn.cpu(),
                                  out=out_w.cpu().to(torch.bfloat16), branch=br)
        self.lay = vo.config_layout(c)
        self.x = x_bf16.cpu()
        self.flops = vo.block_flops(self.lay, c["heads"], c["dim"], c["hidden"])["total"]

    def step(self):
        """One full block forward; returns (output [S, hidden] fp32, seconds)."""
        vo = self.vo
        prev_c, prev_m = vo.set_compute_dtype(torch.float32), vo.set_matmul_dtype(torch.bfloat16)
        try:
            t0 = time.perf_counter()
            out = vo.block_forward(self.x, self.bw, self.lay, self.c["heads"], self.c["dim"], vo.BranchConfig(),
                                   attention="grouped")
            return out, time.perf_counter() - t0
        finally:
            vo.set_compute_dtype(prev_c)
            vo.set_matmul_dtype(prev_m)

    def describe(self, seconds) -> dict:
        return {"cores": self.threads, "cpu": cpu_model(), "kind": "port",
                "sample": f"one full block forward of the config (all {self.c['heads']} heads, {self.lay.seq_len} "
                          f"rows): oracle port of the reference torch path at bf16 GEMM operands, fp32 branch "
                          f"statistics; {seconds:.1f} s for {self.flops / 1e12:.2f} TFLOP"}


def cpu_baseline(c, weights, x_bf16, out_gpu=None):
    """One full block forward on the host cores (``ReferenceCPU``), timed; with ``out_gpu``
    (the GPU block's output for the same weights and input) also the relative L2 between
    the two, the parity figure of the benchmarked output."""
    ref = ReferenceCPU(c, weights, x_bf16)
    out, dt = ref.step()
    line = dict({"value": ref.flops / dt / 1e12, "unit": "TFLOP/s"}, **ref.describe(dt))
    parity = None
    if out_gpu is not None:
        got = out_gpu.double().cpu()
        want = out.double()
        parity = {"rel_l2": float((got - want).norm() / want.norm()), "rows": int(got.shape[0]), "tolerance": 2e-2,
                  "against": "the reference torch path restated on the CPU (bf16 GEMMs, fp32 branch), same "
                             "seeded weights and input, every output row"}
    return line, parity


def make_weights(c, device, seed=0, head_slice=None):
    """Seeded random-init weights of one block (N(0, 0.02) projections), built on device."""
    from oracle import vdn_oracle as vo

    H, D, hidden = c["heads"], c["dim"], c["hidden"]
    g = torch.Generator().manual_seed(seed)
    inner = H * D
    qkv = torch.randn(3 * inner, hidden, generator=g) * 0.02
    out = torch.randn(hidden, inner, generator=g) * 0.02
    qn = 1 + 0.1 * torch.randn(D, generator=g)
    kn = 1 + 0.1 * torch.randn(D, generator=g)
    branch = vo.make_branch_weights(g, hidden, H, D)
    return qkv, qn, kn, out, branch


def bench_input(c):
    """The seed-1 N(0, 1) block input, bf16, on the host."""
    g = torch.Generator().manual_seed(1)
    S = c["text"] + c["frames"] * c["grid"][0] * c["grid"][1]
    return torch.randn(S, c["hidden"], generator=g).to(torch.bfloat16)


def config_entry(args, c, world) -> dict:
    """The ``config`` object of both arms' JSON lines."""
    H, D, hidden = c["heads"], c["dim"], c["hidden"]
    S = c["text"] + c["frames"] * c["grid"][0] * c["grid"][1]
    return {"workload": f"config{args.config}: {c['frames']}x{c['grid'][0] * c['grid'][1]}+{c['text']} tokens, "
                        f"H={H}, D={D}, hidden={hidden}", "tokens": S,
            "parallelism": (f"heads/{world}, exchange {args.exchange}" if world > 1 else "none"),
            "l2": f"inputs larger than L2 (x {S * hidden * 2 / 1e6:.0f} MB, weights "
                  f"{(5 * H * D + 2 * H + 2 * D) * hidden * 2 / 1e9:.2f} GB)",
            "delta_rule": args.delta_rule, "rope": bool(args.rope), "precision": args.precision}


def run_reference_arm(args, c, world, rank):
    """The reference arm: every step is one full block forward of the config on the host
    cores (``ReferenceCPU``), timed by the wall clock; rank 0 alone works and prints."""
    if rank != 0:
        return
    ref = ReferenceCPU(c, make_weights(c, "cpu"), bench_input(c))
    times = []
    for i in range(args.warmup + args.steps):
        _, dt = ref.step()
        if i >= args.warmup:
            times.append(dt)
    times.sort()
    dt = times[len(times) // 2] if times else float("nan")
    val = ref.flops / dt / 1e12
    line = {
        "impl": "reference", "metric": metric_name(c), "value": val, "unit": "TFLOP/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "timed_s": sum(times),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) weights, N(0,1) x)", "config": config_entry(args, c, 1),
        "tflop_per_step": ref.flops / 1e12,
        "cpu_baseline": dict({"value": val, "unit": "TFLOP/s"}, **ref.describe(dt)),
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


E2E_ROW_BLOCKS = 8  # row blocks of the end-to-end copies at N = 1 (4: 15.98 ms e2e, 8: 15.81, 16: 16.23)


def node_config(delta_rule="vdn_solve") -> dict:
    """BASELINE config 1's released-lineage block structure as a node config: short conv on
    k and v, the text state, both gates, the alpha bridge (nodes.py:98-116 keys)."""
    return {"enable_softmax_gate": True, "delta_rule": delta_rule, "bridge": "alpha", "short_conv": ("k", "v"),
            "enable_text_state": True}


def metric_name(c) -> str:
    """BASELINE's metric on the config's geometry (config 1: 31x836+512 tokens)."""
    return (f"VDN hybrid block fwd TFLOP/s at {c['frames']}x{c['grid'][0] * c['grid'][1]}+{c['text']} tokens "
            "(ms in ms_per_step)")


def run_attention_only(args, c):
    """The window attention kernel alone on the config geometry (profiling / roofline)."""
    from __graft_entry__ import load_package
    from oracle import vdn_oracle as vo  # FLOP model only

    pkg = load_package()
    dev = torch.device("cuda", 0)
    H, D = c["heads"], c["dim"]
    lay = pkg.make_layout(c["text"], c["frames"], c["grid"])
    flops = 4.0 * vo.attention_pairs(vo.config_layout(c)) * D * H
    g = torch.Generator().manual_seed(0)
    S = lay.seq_len
    q = torch.randn(S, H, D, generator=g).to(dev, torch.bfloat16)
    k = torch.randn(S, H, D, generator=g).to(dev, torch.bfloat16)
    v = torch.randn(S, H, D, generator=g).to(dev, torch.bfloat16)
    plans = pkg.WindowPlanCache()
    st = pkg._lib.DeviceStatus(dev)
    call = lambda: pkg.window_softmax_b200(q, k, v, lay.video_start, lay.video_end, lay.num_frames,  # noqa: E731
                                           lay.tokens_per_frame, lay.bounds, D ** -0.5, lay.anchor_frames,
                                           cache=plans, status=st)
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        call()
    e1.record()
    torch.cuda.synchronize()
    st.raise_if_failed()
    ms = e0.elapsed_time(e1) / max(args.steps, 1)
    pk, src = peaks()
    print(json.dumps({"kernel": "window_attention_kernel", "heads": H, "tokens": S, "ms": ms,
                      "tflops": flops / (ms * 1e-3) / 1e12, "frac_of_burst_peak": flops / (ms * 1e-3) / 1e12 /
                      pk["bf16_tflops"], "peak_source": src}), flush=True)


def run_quantisers_only(args, c):
    """The activation quantisers alone on the config's branch rows x hidden (bf16, larger than
    L2): plain per-row int8, ConvRot int8 (group-256 rotation in the same pass) and per-tensor
    e4m3 (an amax pass, then the cast), each with the algorithmic bytes of one quantisation
    (2 B read + 1 B written per element, 4 B of scale per row) over its CUDA-event time, against
    the measured HBM copy bandwidth."""
    from __graft_entry__ import load_package

    pkg = load_package()
    dev = torch.device("cuda", 0)
    rows = (c["frames"] - 2) * c["grid"][0] * c["grid"][1]
    K = c["heads"] * c["dim"]
    g = torch.Generator().manual_seed(0)
    x = torch.randn(rows, K, generator=g).to(dev, torch.bfloat16)
    out = pkg.projection.QuantizedMatrix(torch.empty(rows, K, device=dev, dtype=torch.int8),
                                         torch.empty(rows, device=dev, dtype=torch.float32), "int8")
    out8 = pkg.projection.QuantizedMatrix(torch.empty(rows, K, device=dev, dtype=torch.float8_e4m3fn),
                                          torch.empty(1, device=dev, dtype=torch.float32), "fp8")
    work = torch.empty(1, device=dev, dtype=torch.float32)
    pk, src = peaks()
    algo = rows * K * 3 + rows * 4
    for name, fn in (("int8_rows_vec_kernel", pkg.quantize_rows_int8),
                     ("int8_rows_convrot_kernel", pkg.quantize_rows_int8_convrot),
                     ("amax_kernel + fp8_cast_kernel (reads the rows twice)",
                      lambda t, _o: pkg.quantize_tensor_fp8(t, out8, work))):
        for _ in range(args.warmup):
            fn(x, out)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn(x, out)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / max(args.steps, 1)
        gbs = algo / (ms * 1e-3) / 1e9
        print(json.dumps({"kernel": name, "rows": rows, "K": K, "ms": ms, "algorithmic_bytes": algo,
                          "gbs": gbs, "frac_of_hbm": gbs / pk["hbm_gbs"], "peak_source": src}), flush=True)


def run_gemms_only(args, c):
    """The block's QKV projection GEMM alone ([rows, hidden] x [3 H D, hidden]^T, bf16 out) in
    the precision of ``--precision``: bf16 operands (kind 0), per-row int8 codes with row and
    column scales in the epilogue (kind 2), or per-tensor e4m3 with device scales (kind 1).
    ``--rows`` takes a smaller row count for profiling; the operands are quantised once,
    outside the timed launches.  TFLOP/s against the measured bf16 peak (sustained) and, for
    int8 / fp8, against twice it (the dense 8-bit : bf16 ratio of the part, 4.5 : 2.25)."""
    from __graft_entry__ import load_package

    pkg = load_package()
    dev = torch.device("cuda", 0)
    rows = args.rows or (c["text"] + c["frames"] * c["grid"][0] * c["grid"][1])
    hidden, N = c["hidden"], 3 * c["heads"] * c["dim"]
    g = torch.Generator().manual_seed(0)
    x = torch.randn(rows, hidden, generator=g).to(dev, torch.bfloat16)
    w = (torch.randn(N, hidden, generator=g) * 0.02).to(dev, torch.bfloat16)
    out = torch.empty(rows, N, device=dev, dtype=torch.bfloat16)
    if args.precision == "int8":
        xa, wq = pkg.quantize_rows_int8(x), pkg.quantize_rows_int8(w)
        fn = lambda: pkg.gemm(xa.data, wq.data, out=out, row_scale=xa.scale, col_scale=wq.scale, kind=2)
    elif args.precision == "fp8":
        xa, wq = pkg.quantize_tensor_fp8(x), pkg.quantize_tensor_fp8(w)
        fn = lambda: pkg.gemm(xa.data, wq.data, out=out, dev_scale0=xa.scale, dev_scale1=wq.scale, kind=1)
    else:
        fn = lambda: pkg.gemm(x, w, out=out)
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / max(args.steps, 1)
    tflops = 2 * rows * N * hidden / (ms * 1e-3) / 1e12
    pk, src = peaks()
    peak = pk["bf16_tflops_sustained"] * (1 if args.precision == "bf16" else 2)
    print(json.dumps({"kernel": f"gemm_kernel<{ {'bf16': 0, 'fp8': 1, 'int8': 2}[args.precision] }>",
                      "precision": args.precision, "M": rows, "N": N, "K": hidden, "ms": ms, "tflops": tflops,
                      "peak": peak, "frac": tflops / peak,
                      "peak_source": f"{src} bf16 sustained" + ("" if args.precision == "bf16" else " x 2")}),
          flush=True)


def run_convs_only(args, c):
    """The branch's k-feature convolutions alone on the config's clip frames (frames - 2
    frames of the grid, H*D channels): the depthwise 5x5 spatial conv reading the k columns of
    a [rows, 3 H D] QKV buffer, then the 5-tap temporal conv + SiLU + L2 writing [F, H, T, D].
    Each is timed by CUDA events over ``--steps`` launches and reported against its
    algorithmic bytes (2 B read + 2 B written per element) and the measured HBM copy
    bandwidth."""
    from __graft_entry__ import load_package

    pkg = load_package()
    dev = torch.device("cuda", 0)
    gh, gw = c["grid"]
    F, H, D = c["frames"] - 2, c["heads"], c["dim"]
    C, T = H * D, gh * gw
    rows = F * T
    g = torch.Generator().manual_seed(0)
    qkv = torch.randn(rows, 3 * C, generator=g).to(dev, torch.bfloat16)
    k = qkv[:, C:2 * C]
    w_sp = (torch.randn(C, 25, generator=g) * 0.2).to(dev)
    w_tm = (torch.randn(C, 5, generator=g) * 0.45).to(dev)
    sp = torch.empty(rows, C, device=dev, dtype=torch.bfloat16)
    feat = torch.empty(F, H, T, D, device=dev, dtype=torch.bfloat16)
    s = pkg._lib.stream_handle(dev)
    pk, src = peaks()
    algo = rows * C * 4
    for name, fn in (("spatial_conv5_tiled_kernel",
                      lambda: pkg._lib.call("vdn_spatial_conv", k.data_ptr(), k.stride(0), w_sp.data_ptr(), 5, 5, F,
                                            gh, gw, C, sp.data_ptr(), C, s)),
                     ("temporal_act_kernel<128, 5>",
                      lambda: pkg._lib.call("vdn_temporal_act", sp.data_ptr(), C, w_tm.data_ptr(), 5, F, T, H, D, 1,
                                            feat.data_ptr(), s))):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / max(args.steps, 1)
        gbs = algo / (ms * 1e-3) / 1e9
        print(json.dumps({"kernel": name, "frames": F, "grid": [gh, gw], "channels": C, "ms": ms,
                          "algorithmic_bytes": algo, "gbs": gbs, "frac_of_hbm": gbs / pk["hbm_gbs"],
                          "peak_source": src}), flush=True)


def run_dit_stack(args, c, world, rank, local):
    """Config 4: the denoiser forward stack of ``blocks`` DiT blocks (hybrid attention + GELU MLP,
    INT8 projections) over a CFG batch of 2 latent sequences; one step = one sampler step
    (cfg_batch x blocks block forwards).  Weights are random-init on the device, seeded."""
    from __graft_entry__ import load_package
    from oracle import vdn_oracle as vo  # FLOP model only

    pkg = load_package()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    H, D, hidden = c["heads"], c["dim"], c["hidden"]
    F = c["ffn_mult"] * hidden
    n_blocks = args.blocks or c["blocks"]
    lay = pkg.make_layout(c["text"], c["frames"], c["grid"])
    lay_o = vo.config_layout(c)
    S = lay.seq_len
    fl_block = vo.dit_flops(lay_o, H, D, hidden, F, c["activation"])["total"]
    fl_step = fl_block * n_blocks * c["cfg_batch"]
    shard = pkg.shard.default_shard(H) if world > 1 else None
    gen = torch.Generator(device=dev).manual_seed(0)

    def rn(*shape, s=0.02, mean=0.0):
        return torch.randn(*shape, device=dev, dtype=torch.bfloat16, generator=gen) * s + mean

    base_branch = vo.make_branch_weights(torch.Generator().manual_seed(0), hidden, H, D)
    ws_attn, ws_mlp, blocks, mods = {}, {}, [], []
    for _ in range(n_blocks):
        branch = dict(base_branch)
        branch["to_out_linear.weight"] = rn(hidden, H * D)
        if c["precision"] != "bf16":
            # the branch projection runs in its stored representation: store it quantised
            branch = pkg.prepare_projection_maps([branch], dev, c["precision"], skip_end_blocks=0)[0][0]
        fb = pkg.FusedBlock(rn(3 * H * D, hidden), rn(D, s=0.1, mean=1.0), rn(D, s=0.1, mean=1.0), rn(hidden, H * D),
                            branch, H, D, dev, precision=c["precision"], shard=shard, workspaces=ws_attn)
        blocks.append(pkg.B200DiTBlock(fb, rn(hidden, s=0.1, mean=1.0), 1e-6, rn(hidden, s=0.1, mean=1.0), 1e-6,
                                       rn(F, hidden), rn(F), rn(hidden, F), rn(hidden), dev,
                                       activation=c["activation"], precision=c["precision"], workspaces=ws_mlp))
        mods.append([rn(2, hidden, s=0.1, mean=1.0 if name.startswith("gate") else 0.0)
                     for name in pkg.dit.MOD_NAMES])
    group = pkg.dit.segment_indices([(0, lay.video_start, 0), (lay.video_start, S, 1)], S, dev)
    plans = pkg.WindowPlanCache()
    status = pkg.DeviceStatus(dev)
    g = torch.Generator().manual_seed(1)
    x_host = [torch.randn(S, hidden, generator=g).to(torch.bfloat16).pin_memory() for _ in range(c["cfg_batch"])]
    out_host = [torch.empty(S, hidden, dtype=torch.bfloat16).pin_memory() for _ in range(c["cfg_batch"])]
    x_dev = [t.to(dev) for t in x_host]

    def sampler_step(copies=False):
        for i in range(c["cfg_batch"]):
            if copies:
                x_dev[i].copy_(x_host[i], non_blocking=True)
            x = x_dev[i]
            for b, blk in enumerate(blocks):
                x = blk.forward(x, mods[b], group, lay, plans, status)
            if copies:
                out_host[i].copy_(x, non_blocking=True)

    clocks = ClockSampler(local).start()
    with pkg.cholesky_runtime_scope():
        for _ in range(args.warmup):
            sampler_step()
    torch.cuda.synchronize()
    status.raise_if_failed()
    barrier(world)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.mark_start()
    launches0 = pkg._lib.launch_count()
    e0.record()
    with pkg.cholesky_runtime_scope():
        for _ in range(args.steps):
            sampler_step()
        e1.record()
        torch.cuda.synchronize()
    launches = pkg._lib.launch_count() - launches0
    clocks.mark_end()
    barrier(world)
    status.raise_if_failed()
    ms = max_over_ranks(e0.elapsed_time(e1) / max(args.steps, 1), world)
    # end to end: every sampler step copies the CFG batch's latents in from pinned host memory
    # and the denoised outputs back
    barrier(world)
    torch.cuda.synchronize()
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record()
    with pkg.cholesky_runtime_scope():
        for _ in range(args.steps):
            sampler_step(copies=True)
        c1.record()
        torch.cuda.synchronize()
    e2e_ms = max_over_ranks(c0.elapsed_time(c1) / max(args.steps, 1), world)
    clocks.stop()
    status.raise_if_failed()
    pk, pk_src = peaks()
    if rank == 0:
        io_bytes = c["cfg_batch"] * S * hidden * 2
        line = {
            "metric": f"VDN-H3 DiT denoiser TFLOP/s: {n_blocks} blocks x CFG {c['cfg_batch']} per sampler step "
                      f"(ms per sampler step in ms_per_step)",
            "value": fl_step / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int8" if c["precision"] == "int8" else "bf16",
            "data": "synthetic (seeded random-init weights on the device, N(0,1) latents)",
            "config": {"workload": f"config4: {n_blocks} DiT blocks (hybrid attention + {c['activation'].upper()} "
                                   f"{c['ffn_mult']}x MLP, {c['precision']} projections), CFG batch "
                                   f"{c['cfg_batch']}, {c['frames']}x{c['grid'][0] * c['grid'][1]}+{c['text']} tokens",
                       "tokens": S, "blocks": n_blocks, "sampler_steps_timed": args.steps,
                       "parallelism": f"heads sharded over {world} GPUs, MLP token-parallel" if world > 1 else "none",
                       "l2": "every block's weights and activations exceed L2"},
            "tflop_per_step": fl_step / 1e12, "tflop_per_block": fl_block / 1e12,
            "ms_per_block_forward": ms / (n_blocks * c["cfg_batch"]),
            "roofline": {"kernel": "whole denoiser step", "bound": "tensor",
                         "achieved": fl_step / (ms * 1e-3) / 1e12 / world, "peak": pk.get("bf16_tflops_sustained"),
                         "unit": "TFLOP/s per GPU", "frac": fl_step / (ms * 1e-3) / 1e12 / world /
                         pk.get("bf16_tflops_sustained", 1.0), "traffic": None,
                         "peak_source": f"{pk_src} sustained bf16 (int8 tensor peak is 2x)"},
            "e2e": {"value": fl_step / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": io_bytes, "d2h_bytes_per_step": io_bytes},
            "gpu_launches": launches,
            "clocks": clocks.summary(),
        }
        print(json.dumps(line), flush=True)


def rope_freqs_table(seq, rot, dev):
    """A [1, seq, 1, rot/2, 2, 2] RoPE table of 1-D positions (ComfyUI's layout), built on the device."""
    pos = torch.arange(seq, device=dev, dtype=torch.float64)
    omega = 1.0 / 10000.0 ** (torch.arange(0, rot, 2, device=dev, dtype=torch.float64) / rot)
    ang = pos[:, None] * omega[None]
    c, s_ = torch.cos(ang), torch.sin(ang)
    m = torch.stack([torch.stack([c, -s_], -1), torch.stack([s_, c], -1)], -2).float()
    return m.reshape(1, seq, 1, rot // 2, 2, 2)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200")
    ap.add_argument("--config", type=int, default=1)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--only", choices=["attention", "quantisers", "gemms", "convs"], default=None,
                    help="run one kernel alone on the config geometry (profiling small cases)")
    ap.add_argument("--heads", type=int, default=None, help="override the head count (profiling small cases)")
    ap.add_argument("--rows", type=int, default=None, help="--only gemms: row count (profiling small cases)")
    ap.add_argument("--e2e-blocks", type=int, default=E2E_ROW_BLOCKS,
                    help="row blocks per host copy in the end-to-end leg at N = 1")
    ap.add_argument("--blocks", type=int, default=None, help="config 4: number of DiT blocks (default 50)")
    ap.add_argument("--delta-rule", choices=["vdn_solve", "sana_scaled"], default="vdn_solve",
                    help="configs 1/3: the branch's delta rule (BASELINE's released lineage is vdn_solve)")
    ap.add_argument("--exchange", choices=["rows", "heads"], default="rows",
                    help="N > 1: all-to-all by row block + row-split projection (rows) or all-gather of the "
                         "per-head outputs + projection on every GPU (heads)")
    ap.add_argument("--precision", choices=["bf16", "int8", "fp8"], default="bf16",
                    help="configs 1/3: projection arithmetic (config 2 = config 1 with int8 or fp8)")
    ap.add_argument("--rope", action="store_true",
                    help="configs 1/3: apply a rot_dim = head_dim RoPE table to q/k (not in BASELINE's config)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup()
    c = dict(CONFIGS[args.config])
    if args.heads:
        c["heads"] = args.heads
    if args.only == "attention":
        run_attention_only(args, c)
        return
    if args.only == "quantisers":
        run_quantisers_only(args, c)
        return
    if args.only == "gemms":
        run_gemms_only(args, c)
        return
    if args.only == "convs":
        run_convs_only(args, c)
        return
    if args.config == 4 and args.impl != "reference":
        run_dit_stack(args, c, world, rank, local)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    if args.impl == "reference":
        run_reference_arm(args, c, world, rank)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return

    from __graft_entry__ import _Attn, load_package
    from oracle import vdn_oracle as vo  # FLOP model only (no oracle compute on this path)

    pkg = load_package()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    H, D, hidden = c["heads"], c["dim"], c["hidden"]
    lay = pkg.make_layout(c["text"], c["frames"], c["grid"])
    lay_o = vo.config_layout(c)
    flops = vo.block_flops(lay_o, H, D, hidden)
    qkv, qn, kn, out_w, branch = make_weights(c, dev)
    import types

    attn = types.SimpleNamespace(heads=H, head_dim=D, qkv_proj=types.SimpleNamespace(weight=qkv),
                                 out_proj=types.SimpleNamespace(weight=out_w),
                                 q_norm=types.SimpleNamespace(weight=qn, eps=1e-6),
                                 k_norm=types.SimpleNamespace(weight=kn, eps=1e-6), forward=None)
    # N > 1: the heads are sharded over the ranks (H/N each, recurrence kept per head), the
    # per-head outputs exchanged by row block over NCCL and the projected rows all-gathered
    maps = None
    if args.precision != "bf16":
        # config 2: qkv_proj / out_proj quantised by the block, to_out_linear stored quantised
        # (no bf16 edge block: the benchmarked block is an interior one)
        maps = pkg.prepare_projection_maps([branch], dev, args.precision, skip_end_blocks=0)[0]
    state = pkg.B200State("bench", node_config(args.delta_rule), [branch], H, D, shard_heads=world > 1,
                          projection_precision=args.precision, weight_maps=maps, shard_exchange=args.exchange)
    block = state.fused_block(attn, 0, dev)
    rope_freqs = rope_freqs_table(lay.seq_len, D, dev) if args.rope else None
    rope = pkg.rope_table(rope_freqs, lay.seq_len, D, dev)
    status = state.device_status(dev)
    x_host = bench_input(c).pin_memory()
    x_dev = x_host.to(dev)
    out_dev = torch.empty(lay.seq_len, hidden, device=dev, dtype=torch.bfloat16)
    # ---- device-resident timing (inputs in HBM; x 270 MB and weights ~0.3 GB exceed the 126 MB L2)
    attn_ms = []
    orig_launch = pkg.hybrid.launch_window_attention

    def timed_launch(*a, **k):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        orig_launch(*a, **k)
        e1.record()
        attn_ms.append((e0, e1))

    pkg.hybrid.launch_window_attention = timed_launch
    # the projection GEMMs' own launches, timed the same way (their streams are the current one)
    gemm_ms = {"vdn_qkv_gemm": [], "vdn_gemm_block": []}
    orig_call = pkg._lib.call

    def timed_call(name, *a):
        if name not in gemm_ms:
            return orig_call(name, *a)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        orig_call(name, *a)
        e1.record()
        gemm_ms[name].append((e0, e1))

    pkg._lib.call = timed_call
    clocks = ClockSampler(local).start()  # running through the warm-up, so it samples the timed region
    with pkg.cholesky_runtime_scope():
        for _ in range(args.warmup):
            block.forward(x_dev, lay, state.window_plans, status, out=out_dev if world == 1 else None, rope=rope)
    torch.cuda.synchronize()
    status.raise_if_failed()
    attn_ms.clear()
    for v in gemm_ms.values():
        v.clear()
    barrier(world)
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clocks.mark_start()
    launches0 = pkg._lib.launch_count()
    e_start.record()
    with pkg.cholesky_runtime_scope():
        for _ in range(args.steps):
            block.forward(x_dev, lay, state.window_plans, status, out=out_dev if world == 1 else None, rope=rope)
        e_end.record()
        torch.cuda.synchronize()
    clocks.mark_end()
    launches = pkg._lib.launch_count() - launches0  # this library's kernels in the timed region
    barrier(world)
    status.raise_if_failed()
    pkg.hybrid.launch_window_attention = orig_launch
    pkg._lib.call = orig_call
    ms = e_start.elapsed_time(e_end) / max(args.steps, 1)
    ms = max_over_ranks(ms, world)
    value = flops["total"] / (ms * 1e-3) / 1e12  # one block forward of the whole problem per step
    # the attention of one forward may be several launches (one per row chunk when the heads
    # are sharded and the exchange is chunked): sum them per step
    attn_avg = sum(a.elapsed_time(b) for a, b in attn_ms) / max(args.steps, 1)
    attn_launches = len(attn_ms) // max(args.steps, 1)
    pk, pk_src = peaks()
    achieved = flops["attention"] / world / (attn_avg * 1e-3) / 1e12  # this rank's heads
    peak = pk.get("bf16_tflops_sustained", pk["bf16_tflops"])
    # projection GEMMs per forward: the QKV GEMM (its algorithmic q/k/v columns) and the output
    # projection passes (out_proj + to_out_linear), against the tensor peak of their arithmetic
    # (int8 / e4m3 run at twice the bf16 rate: the measured bf16 peak doubled)
    steps_n = max(args.steps, 1)
    qkv_ms = sum(a.elapsed_time(b) for a, b in gemm_ms["vdn_qkv_gemm"]) / steps_n
    out_ms = sum(a.elapsed_time(b) for a, b in gemm_ms["vdn_gemm_block"]) / steps_n
    gemm_peak = peak * (1 if args.precision == "bf16" else 2)
    gemm_line = {}
    for name, fl, t in (("qkv", flops["qkv"] / world, qkv_ms),
                        ("out_proj+to_out_linear", flops["out_proj"] + flops.get("to_out_linear", 0.0), out_ms)):
        if t > 0:
            gemm_line[name] = {"ms": t, "achieved": fl / (t * 1e-3) / 1e12, "peak": gemm_peak, "unit": "TFLOP/s",
                               "frac": fl / (t * 1e-3) / 1e12 / gemm_peak}
    gemm_line["peak_source"] = (f"{pk_src} sustained bf16" if args.precision == "bf16" else
                                f"2 x {pk_src} sustained bf16 (dense {args.precision} tensor rate)")
    # ---- end to end through the public operator with host buffers: every step copies its
    # input from pinned host memory and its output back; HostStreamer overlaps the copies of
    # steps i+1 and i-1 with the compute of step i
    fwd = pkg.make_vdn_forward(attn, state, 0)
    S = lay.seq_len

    def run_fwd(xd, io=None):
        with pkg.publish_layout(lay):
            return fwd(xd, rope_freqs,
                       transformer_options={pkg.hybrid.STREAM_IO_KEY: io} if io is not None else None)

    if world == 1:
        streamer = pkg.HostStreamer(run_fwd, dev, (S, hidden))
        inputs_host = [x_host]
        outs_host = [torch.empty(S, hidden, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
        prepare = None
    else:
        # each rank holds its own row block of x and of the output in pinned host memory:
        # H2D of the block, NCCL all-gather of x, sharded forward, D2H of the rank's rows
        import torch.distributed as dist

        sb = -(-S // world)
        r0, n_rows = rank * sb, max(0, min(sb, S - rank * sb))
        x_rows_host = torch.zeros(sb, hidden, dtype=torch.bfloat16).pin_memory()
        x_rows_host[:n_rows] = x_host[r0:r0 + n_rows]
        x_all = torch.empty(world * sb, hidden, device=dev, dtype=torch.bfloat16)

        def prepare(xr):
            dist.all_gather_into_tensor(x_all, xr)
            return x_all[:S]

        streamer = pkg.HostStreamer(lambda xd: run_fwd(xd)[r0:r0 + n_rows], dev, (sb, hidden))
        inputs_host = [x_rows_host]
        outs_host = [torch.empty(n_rows, hidden, dtype=torch.bfloat16).pin_memory() for _ in range(2)]

    def e2e_run(k):
        # one GPU: inputs copied in and outputs copied back by row blocks, overlapping the
        # first step's QKV and the last step's output projection too
        streamer.run([inputs_host[0]] * k, [outs_host[i & 1] for i in range(k)], prepare=prepare,
                     chunks=args.e2e_blocks if world == 1 else 1)

    # warm up the way the timed steps run: inside one status scope, so every forward is
    # validated at the scope's end and none waits for the host in between
    with pkg.cholesky_runtime_scope():
        e2e_run(args.warmup)
        torch.cuda.synchronize()
    barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with pkg.cholesky_runtime_scope():
        e0.record(streamer.h2d)  # before the first input copy
        e2e_run(args.steps)
        torch.cuda.current_stream(dev).wait_stream(streamer.d2h)
        e1.record()  # after the last output copy
        torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / max(args.steps, 1), world)
    status.raise_if_failed()
    # diagnostics outside the timed region: one bare host->device and device->host copy
    c0, c1, c2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    x_probe = torch.empty_like(streamer.x_dev[0])
    c0.record()
    x_probe.copy_(inputs_host[0], non_blocking=True)
    c1.record()
    outs_host[0].copy_(x_probe[:outs_host[0].shape[0], :outs_host[0].shape[1]], non_blocking=True)
    c2.record()
    torch.cuda.synchronize()
    copy_ms = {"h2d_ms": c0.elapsed_time(c1), "d2h_ms": c1.elapsed_time(c2)}
    clocks.stop()
    clock_summary = clocks.summary()
    e2e_value = flops["total"] / (e2e_ms * 1e-3) / 1e12
    line = {
        "metric": metric_name(c), "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": args.precision, "data": "synthetic (seeded N(0,0.02) weights, N(0,1) x)",
        "config": config_entry(args, c, world),
        "tflop_per_step": flops["total"] / 1e12,
        "roofline": {"kernel": "window_attention_kernel", "bound": "tensor", "achieved": achieved, "peak": peak,
                     "unit": "TFLOP/s", "frac": achieved / peak,
                     "traffic": attention_traffic(H // world, H) if args.config == 1 else None,
                     "algorithmic_bytes": lay.seq_len * (H // world) * D * 2 * 4, "peak_source": f"{pk_src} sustained",
                     "kernel_ms": attn_avg, "launches_per_step": attn_launches, "block_frac": value / world / peak},
        # bytes summed over the ranks (at N > 1 each rank moves its own row block)
        "e2e": {"value": e2e_value, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": S * hidden * 2, "d2h_bytes_per_step": S * hidden * 2,
                "copies": "pinned host buffers; H2D of step i+1 and D2H of step i-1 overlap step i (HostStreamer); "
                  f"{args.e2e_blocks if world == 1 else 1} row blocks per copy",
                **copy_ms},
        "gpu_launches": launches,
        "gemm": gemm_line,
        "clocks": clock_summary,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline and args.precision == "bf16":
        # the same block on the host cores: the CPU baseline, and the parity of the benchmarked
        # output (out_dev holds the last device-resident step's output for x)
        baseline, parity = cpu_baseline(c, (qkv, qn, kn, out_w, branch), x_host,
                                        out_dev if not args.rope else None)
        line["cpu_baseline"] = baseline
        if parity is not None:
            line["parity_rel_l2"] = parity["rel_l2"]
            line["parity"] = parity
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
