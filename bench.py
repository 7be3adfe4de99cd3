#!/usr/bin/env python
"""Benchmark of the KaniTTS fused decode-path kernels on B200.

Headline workload (one "step" = one launch of the fused kernel):
  rope_kv_write, bf16: T = 4096 tokens of Q [T, 16, 64], K/V [T, 8, 64]
  ~ N(0, 1); rotary theta = 1e6 with the learnable alpha at its init
  (w = 0 -> alpha = 1.05 in bf16); positions 0..4095; frame table
  [1024, 64] ~ N(0, 0.02) indexed by position // 4; K/V written into a
  static cache [1, 8, 4096, 64] at slot = position.  This is the prefill
  end of the decode-step RoPE + KV-write configuration (its sweep maximum).
  Eight independent input sets (272 MB > 126 MB L2) rotate between steps, so
  every step reads cold inputs from HBM.

  metric: fused-op HBM GB/s = algorithmic bytes / time, 8320 B per token
  (read Q 2048 + K 1024 + V 1024 + frame row 128, write Q 2048 + K slot
  1024 + V slot 1024).

Timing: W warm-up launches, then exactly K launches replayed from CUDA
graphs, bracketed by a barrier + synchronize; the CUDA events that time them
are recorded inside the graphs on the launching stream, after 8 untimed
lead-in launches, so the host's graph submission is outside the timed
region.  The max over ranks is taken.  N > 1 runs N independent
replicas (the work shards by independent streams; there is no collective on
the data path), so scaling is weak.

Also reported:
  e2e         — the same metric through the public Python API with pinned host
                buffers: per step H2D of Q/K/V/positions/slots, the kernel, and
                D2H of the rotated Q and the written K/V slots;
  roofline    — achieved vs the measured HBM copy peak (MEASURED_PEAKS.json),
                with the steady-state DRAM traffic per launch from the committed
                ncu summary;
  cpu_baseline— the CPU oracle (PyTorch eager restatement of the reference
                path) on the host cores, rank 0 at N = 1;
  sweep       — every fused op at its configuration sizes (µs per call and GB/s),
                next to the reference's own Triton kernels on the same GPU and
                inputs when the reference is installed in baseline/_ref;
  decode      — the synthetic LFM2 decode step on the fused kernels: bs=1 and 64
                streams per GPU (tokens/s aggregated over the N GPUs), greedy and
                sampled, and at bs=1 the reference's own Triton + CUDA-graph
                engine (OptimizedDecoder captured by KaniInferenceEngine) on the
                same GPU, with its greedy tokens compared to this library's;
  clocks      — nvidia-smi samples taken during the timed region.

``--impl reference`` times the reference's CPU path (the oracle port: the
reference's decode path has no CPU implementation besides the eager ops the
oracle restates) on the same workload and prints the same line with
"impl": "reference".  Rank 0 alone runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "kani-tts-2-openai-server_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "fused-op HBM GB/s vs peak; decode step µs & tokens/s (LFM2-style, bs=1/64)"
UNIT = "GB/s"
T_TOK, HQ, HK, D = 4096, 16, 8, 64
TABLE_ROWS, TPF = 1024, 4
BYTES_PER_TOKEN = 8320
STEP_BYTES = BYTES_PER_TOKEN * T_TOK
N_SETS = 8
WORKLOAD = (f"rope_kv_write bf16 T={T_TOK} Q[{T_TOK},{HQ},{D}] K/V[{T_TOK},{HK},{D}] theta=1e6 alpha=1.05 "
            f"frame_table[{TABLE_ROWS},{D}] cache[1,{HK},{T_TOK},{D}] slot=pos")


def _peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return 6650.0, "fallback"


def _traffic_per_launch() -> tuple[float | None, str | None]:
    """Steady-state DRAM bytes (read + write) per headline launch, from the
    committed summary of one ncu capture of back-to-back launches with the
    cache left warm between them (profiles/rope_kv_write_t4096_traffic.json)."""
    p = ROOT / "profiles" / "rope_kv_write_t4096_traffic.json"
    if not p.exists():
        return None, None
    try:
        d = json.loads(p.read_text())
        return float(d["steady_state_bytes_per_launch"]), "profiles/rope_kv_write_t4096_traffic.json"
    except (ValueError, KeyError):
        return None, None


def _ref_unavailable(args) -> str:
    if args.no_reference_gpu:
        return "skipped (--no-reference-gpu)"
    from baseline import reference as R
    return R.why_unavailable()


# ------------------------------------------------------------ distributed

def _dist_init():
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


def _barrier(world):
    if world > 1:
        from kani_tts_b200.replicas import barrier
        barrier()


def _gather_over_ranks(x: float, world: int, dev) -> list[float]:
    if world == 1:
        return [x]
    from kani_tts_b200.replicas import gather_over_ranks
    return gather_over_ranks(x, dev)


def _max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    from kani_tts_b200.replicas import max_over_ranks
    return max_over_ranks(x, dev)


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi sampling of one GPU while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, dev: torch.device):
        self.proc = None
        self.lines: list[str] = []
        try:
            uuid = str(torch.cuda.get_device_properties(dev).uuid)
            self.target = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        except Exception:
            self.target = None

    def __enter__(self):
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"]
        if self.target:
            cmd += ["-i", self.target]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
            time.sleep(0.2)
        except (FileNotFoundError, OSError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.reader.join(timeout=5)

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------- workload

def make_inputs(seed: int, t: int = T_TOK, device="cpu"):
    """One seeded input set of the headline workload (generated on the CPU)."""
    from kani_tts_b200 import positions as P
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(t, HQ, D, generator=g).to(torch.bfloat16)
    k = torch.randn(t, HK, D, generator=g).to(torch.bfloat16)
    v = torch.randn(t, HK, D, generator=g).to(torch.bfloat16)
    rows = max(TABLE_ROWS, (t + TPF - 1) // TPF)   # every position has a frame row (T > 4096 too)
    table = (0.02 * torch.randn(rows, D, generator=g)).to(torch.bfloat16)
    inv = P.learnable_inv_freq(D, 1e6, 0.0)
    pos = torch.arange(t, dtype=torch.long)
    s_len = max(2048, t)
    kc = torch.zeros(1, HK, s_len, D, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    d = dict(q=q, k=k, v=v, table=table, inv=inv, pos=pos, slots=pos.clone(), kc=kc, vc=vc)
    return {n: x.to(device) for n, x in d.items()}


def launch(K, s: dict, q_out=None):
    t = s["q"].shape[0]
    return K.fused_rope_kv_write(
        s["q"].view(1, t, HQ, D), s["k"].view(1, t, HK, D), s["v"].view(1, t, HK, D), s["inv"], s["pos"],
        s["kc"], s["vc"], s["slots"], frame_table=s["table"], tokens_per_frame=TPF, q_out=q_out)


def graph_of(fn_list):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for fn in fn_list:
            fn()
    return g


def time_graph_steps(step_fns, steps: int, dev, world: int, chunk: int = 1000, lead: int = 8):
    """Replay exactly `steps` launches (cycling step_fns) from CUDA graphs and
    return the device time of those launches on this rank, in seconds.

    The start and end events are recorded inside the captured graphs (event
    record nodes): the first graph runs `lead` untimed launches, records the
    start event on a branch forked after them (so the timed launches stay
    chained to the lead-in launch by launch, programmatic edges included),
    then its share of the timed launches; the last graph ends with the end
    event.  The host's graph submission and the graph's own
    launch latency therefore stay outside the timed region, however few
    launches it holds."""
    n = len(step_fns)
    chunk = max(1, min(chunk, steps))
    e0 = torch.cuda.Event(enable_timing=True, external=True)
    e1 = torch.cuda.Event(enable_timing=True, external=True)

    def body(first, count):
        for i in range(first, first + count):
            step_fns[i % n]()

    def capture(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        return g

    first = min(chunk, steps)
    full_rest = steps - first
    mids, rest = divmod(full_rest, chunk)
    side = torch.cuda.Stream(device=dev)

    def g_first_body():
        body(0, lead)
        # the start event on a forked branch: it fires when the lead-in completes,
        # and the first timed launch keeps its programmatic edge to the last
        # lead-in launch (an event node between them would break that edge)
        main = torch.cuda.current_stream(dev)
        side.wait_stream(main)
        with torch.cuda.stream(side):
            e0.record(side)
        body(lead, first)
        main.wait_stream(side)
        if full_rest == 0:
            e1.record()
    graphs = [capture(g_first_body)]
    g_mid = capture(lambda: body(lead + first, chunk)) if mids else None
    g_last = None
    if full_rest:
        def g_last_body():
            body(lead + first + mids * chunk, rest)
            e1.record()
        g_last = capture(g_last_body)
    seq = graphs + [g_mid] * mids + ([g_last] if g_last is not None else [])
    for g in {id(g): g for g in seq}.values():   # the first replay uploads each graph
        g.replay()
    torch.cuda.synchronize(dev)
    _barrier(world)
    torch.cuda.synchronize(dev)
    for g in seq:
        g.replay()
    torch.cuda.synchronize(dev)
    _barrier(world)
    return e0.elapsed_time(e1) / 1e3


# ------------------------------------------------------------ CPU arm

def cpu_oracle_rate(seconds: float = 10.0, t: int = T_TOK, max_iters: int | None = None) -> dict:
    """Time the oracle (CPU restatement of the reference path) on host cores."""
    from oracle import kani_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    s = make_inputs(0, t)
    def one():
        kc, vc = s["kc"], s["vc"]
        O.rope_kv_write_ref(s["q"], s["k"], s["v"], s["inv"], s["pos"], kc, vc, s["slots"],
                            frame_table=s["table"], tokens_per_frame=TPF)
    one()
    n, t0 = 0, time.perf_counter()
    while True:
        one()
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or (max_iters is not None and n >= max_iters):
            break
    return {"value": n * BYTES_PER_TOKEN * t / el / 1e9, "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port", "seconds": el, "iters": n,
            "sample": f"{n} oracle calls of the full workload (T={t}) in {el:.1f} s"}


def run_reference(args, world, rank):
    if rank != 0:
        return
    from oracle import kani_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    s = make_inputs(0)
    def one():
        O.rope_kv_write_ref(s["q"], s["k"], s["v"], s["inv"], s["pos"], s["kc"], s["vc"], s["slots"],
                            frame_table=s["table"], tokens_per_frame=TPF)
    for _ in range(args.warmup):
        one()
    steps = min(args.steps, 50)          # bounded sample: each step is the full T=4096 workload
    t0 = time.perf_counter()
    for _ in range(steps):
        one()
    el = time.perf_counter() - t0
    value = steps * STEP_BYTES / el / 1e9
    line = {"metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "ms_per_step": round(el / steps * 1e3, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) inputs)", "impl": "reference",
            "config": {"workload": WORKLOAD, "implementation": "CPU oracle (PyTorch eager restatement of "
                       "kani_tts triton_kernels / optimized_decode / static_cache)", "l2": "n/a (CPU)"},
            "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": torch.get_num_threads(),
                             "kind": "port", "sample": f"{steps} full-workload steps"},
            "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- GPU arm

def run_e2e(K, dev, steps: int) -> dict:
    """Public API with pinned host buffers, every step: H2D of the step's inputs
    (Q, K, V, positions, slots), the kernel, D2H of its results (rotated Q and
    the written K/V cache slots).  The inputs travel as one packed host buffer,
    [T, Q | K | V] rows as the QKV projection lays them out plus the positions
    and slots, read in place through token strides; the results land in one
    device buffer (rotated Q, then the K and V caches, whose every slot this step
    writes).  So a step is one H2D copy, the kernel and one D2H copy.  Steps are
    pipelined over two buffer sets and three streams (copy-in, compute,
    copy-out) so that one step's H2D overlaps the previous step's D2H (PCIe is
    full duplex); events order every buffer reuse."""
    host = make_inputs(1)
    t = T_TOK
    row = (HQ + 2 * HK) * D
    qkv_bytes = t * row * 2
    in_bytes = qkv_bytes + 2 * t * 8
    s_len = host["kc"].shape[2]
    if s_len != t:
        raise RuntimeError("the e2e leg reads the whole cache back: it needs cache length = tokens")
    q_bytes = t * HQ * D * 2
    out_bytes = q_bytes + 2 * HK * s_len * D * 2

    def in_views(buf):
        qkv = buf[:qkv_bytes].view(torch.bfloat16).view(t, row)
        ps = buf[qkv_bytes:in_bytes].view(torch.int64).view(2, t)
        return (qkv[:, :HQ * D].view(1, t, HQ, D), qkv[:, HQ * D:(HQ + HK) * D].view(1, t, HK, D),
                qkv[:, (HQ + HK) * D:].view(1, t, HK, D), ps[0], ps[1])

    def out_views(buf):
        q_out = buf[:q_bytes].view(torch.bfloat16).view(1, t, HQ, D)
        kv = buf[q_bytes:].view(torch.bfloat16).view(2, 1, HK, s_len, D)
        return q_out, kv[0], kv[1]

    pin_in = torch.empty(in_bytes, dtype=torch.uint8).pin_memory()
    q_h, k_h, v_h, pos_h, slots_h = in_views(pin_in)
    q_h.copy_(host["q"].view(1, t, HQ, D))
    k_h.copy_(host["k"].view(1, t, HK, D))
    v_h.copy_(host["v"].view(1, t, HK, D))
    pos_h.copy_(host["pos"])
    slots_h.copy_(host["slots"])
    nbuf = 2
    d_in = [torch.empty(in_bytes, dtype=torch.uint8, device=dev) for _ in range(nbuf)]
    d_out = [torch.zeros(out_bytes, dtype=torch.uint8, device=dev) for _ in range(nbuf)]
    h_out = [torch.empty(out_bytes, dtype=torch.uint8).pin_memory() for _ in range(nbuf)]
    table, inv = host["table"].to(dev), host["inv"].to(dev)
    s_in, s_comp, s_out = (torch.cuda.Stream(device=dev) for _ in range(3))
    ev = lambda: torch.cuda.Event()  # noqa: E731
    in_done = [ev() for _ in range(nbuf)]
    comp_done = [ev() for _ in range(nbuf)]
    out_done = [ev() for _ in range(nbuf)]
    used = [False] * nbuf

    def step(i):
        j = i % nbuf
        with torch.cuda.stream(s_in):
            if used[j]:
                s_in.wait_event(comp_done[j])      # inputs of buffer j no longer read
            d_in[j].copy_(pin_in, non_blocking=True)
            in_done[j].record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(in_done[j])
            if used[j]:
                s_comp.wait_event(out_done[j])     # results of buffer j already read back
            q, k, v, pos, slots = in_views(d_in[j])
            q_out, kc, vc = out_views(d_out[j])
            K.fused_rope_kv_write(q, k, v, inv, pos, kc, vc, slots, frame_table=table, tokens_per_frame=TPF,
                                  q_out=q_out)
            comp_done[j].record(s_comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(comp_done[j])
            h_out[j].copy_(d_out[j], non_blocking=True)
            out_done[j].record(s_out)
        used[j] = True

    for i in range(4):
        step(i)
    torch.cuda.synchronize(dev)
    # the packed path returns what the headline launch computes from contiguous inputs
    ref = make_inputs(1, device=dev)
    ref_q = torch.empty(1, t, HQ, D, dtype=torch.bfloat16, device=dev)
    launch(K, ref, ref_q)
    got_q, got_k, got_v = out_views(h_out[0])
    if not (torch.equal(got_q, ref_q.cpu()) and torch.equal(got_k, ref["kc"].cpu())
            and torch.equal(got_v, ref["vc"].cpu())):
        raise RuntimeError("the packed e2e path differs from the headline launch")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    for i in range(steps):
        step(i)
    s_out.wait_stream(s_in)
    s_out.wait_stream(s_comp)
    e1.record(s_out)
    torch.cuda.synchronize(dev)
    el = e0.elapsed_time(e1) / 1e3
    return {"seconds": el, "steps": steps, "h2d": in_bytes, "d2h": out_bytes}


def host_link_copies(dev, in_bytes: int, out_bytes: int, steps: int) -> float:
    """The host link's share of the e2e leg: the same per-step copies (one pinned
    H2D of `in_bytes`, one D2H of `out_bytes`), pipelined the same way over two
    buffer sets and copy-in / copy-out streams, with no kernel between them.
    Seconds for `steps` steps: the time the e2e leg would take if the kernel
    cost nothing (each rank measures its own, so at N > 1 it shows what the
    GPUs sharing one host get)."""
    nbuf = 2
    h_in = torch.empty(in_bytes, dtype=torch.uint8).pin_memory()
    h_out = [torch.empty(out_bytes, dtype=torch.uint8).pin_memory() for _ in range(nbuf)]
    d_in = [torch.empty(in_bytes, dtype=torch.uint8, device=dev) for _ in range(nbuf)]
    d_out = [torch.zeros(out_bytes, dtype=torch.uint8, device=dev) for _ in range(nbuf)]
    s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    in_done = [torch.cuda.Event() for _ in range(nbuf)]
    out_done = [torch.cuda.Event() for _ in range(nbuf)]
    used = [False] * nbuf

    def step(i):
        j = i % nbuf
        with torch.cuda.stream(s_in):
            if used[j]:
                s_in.wait_event(out_done[j])
            d_in[j].copy_(h_in, non_blocking=True)
            in_done[j].record(s_in)
        with torch.cuda.stream(s_out):
            s_out.wait_event(in_done[j])
            h_out[j].copy_(d_out[j], non_blocking=True)
            out_done[j].record(s_out)
        used[j] = True

    for i in range(4):
        step(i)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s_in)
    for i in range(steps):
        step(i)
    s_out.wait_stream(s_in)
    e1.record(s_out)
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / 1e3


def _ref_cache(ref, dev, s_len: int = 2048):
    """The reference's StaticLfm2HybridConvCache for one attention layer of the
    decode shapes (16 Q heads, 8 KV heads, head_dim 64)."""
    import types as _t
    cfg = _t.SimpleNamespace(num_key_value_heads=HK, head_dim=D, num_hidden_layers=1, hidden_size=HQ * D,
                             num_attention_heads=HQ, layer_types=["full_attention"], conv_L_cache=3)
    return ref.static_cache.StaticLfm2HybridConvCache(cfg, max_total_len=s_len, batch_size=1,
                                                      dtype=torch.bfloat16, device=dev)


def _ref_rope_kv_step(ref, q, k, v, inv, pos, cache, qw=None, kw=None):
    """The reference's RoPE + KV write of one decode token (optimized_decode.py:
    220-240): optional q/k norm (Triton), cos/sin from inv_freq * position with
    eager ops, the two Triton RoPE launches, and the cache's scatter_ update."""
    tk = ref.triton_kernels
    if qw is not None:
        q = tk.fused_rms_norm(q, qw, 1e-5)
        k = tk.fused_rms_norm(k, kw, 1e-5)
    q = q.reshape(1, HQ, 1, D)
    k = k.reshape(1, HK, 1, D)
    freqs = inv * pos[0].float()
    emb = torch.cat([freqs, freqs])
    cos, sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
    q, k = tk.fused_rope(q, k, cos, sin)
    return q, cache.update(k, v.reshape(1, HK, 1, D), 0)


def _triton_rms(ref, x, w, y, eps):
    """The reference's ``_rms_norm_kernel`` launched as ``fused_rms_norm`` launches it
    (triton_kernels.py:49-59), into a given output."""
    import triton
    n = x.shape[-1]
    ref.triton_kernels._rms_norm_kernel[(x.numel() // n,)](x, w, y, N=n, eps=eps, BLOCK_N=triton.next_power_of_2(n))


def _triton_silu(ref, x, y):
    """The reference's ``_silu_mul_kernel`` launched as ``fused_silu_mul`` launches it
    (triton_kernels.py:94-103), into a given output."""
    import triton
    n = x.shape[-1] // 2
    ref.triton_kernels._silu_mul_kernel[(x.numel() // (2 * n),)](x, y, N=n, BLOCK_N=triton.next_power_of_2(n))


def run_sweep(K, dev, peak: float, ref=None) -> dict:
    """Every fused op at its configuration sizes, graph-replayed, inputs rotated.
    With the reference installed (``ref``), its own Triton kernels run on the same
    inputs as a second column: ``triton_us`` / ``triton_GB_s`` (the same
    algorithmic bytes).  They are launched as the reference's wrappers launch
    them (grid, block size) but write into the same rotated output buffers as
    this library's kernels: the wrappers' fresh ``torch.empty`` output would,
    inside a CUDA graph, reuse one pooled address every launch and stay in L2,
    which the rotated outputs here do not."""
    out = {}
    g = torch.Generator().manual_seed(5)
    tk = ref.triton_kernels if ref is not None else None

    def rot_sets(make, nbytes):
        n = int(min(64, max(1, -(-256e6 // max(nbytes, 1)))))
        return [make(i) for i in range(n)]

    def time_us(fns, launches):
        torch.cuda.synchronize(dev)
        g_ = graph_of([fns[i % len(fns)] for i in range(launches)])
        g_.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g_.replay()                     # lead-in: the timed replay is queued while it runs
        e0.record()
        g_.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        del g_
        return e0.elapsed_time(e1) * 1e3 / launches

    def measure(name, sets, nbytes, launches=400):
        us = time_us([s[0] for s in sets], launches)
        gbs = nbytes / (us * 1e-6) / 1e9
        row = {"us": round(us, 3), "GB_s": round(gbs, 1), "frac": round(gbs / peak, 4),
               "bytes": int(nbytes), "rotated_sets": len(sets)}
        if sets[0][1] is not None:
            tus = time_us([s[1] for s in sets], launches)
            row["triton_us"] = round(tus, 3)
            row["triton_GB_s"] = round(nbytes / (tus * 1e-6) / 1e9, 1)
            row["speedup_vs_triton"] = round(tus / us, 3)
        out[name] = row

    # add + RMSNorm (config 1, the 64-stream decode shape, and a row sweep); the
    # reference's composition is the eager add then the Triton norm
    # (optimized_decode.py:252 + :280); its fp32 output holds bf16-rounded values
    for dtype, rows in [(torch.float32, 8), (torch.bfloat16, 1), (torch.bfloat16, 64), (torch.bfloat16, 16384),
                        (torch.bfloat16, 65536), (torch.float32, 16384)]:
        es = torch.tensor([], dtype=dtype).element_size()
        nbytes = rows * 1024 * es * 4 + 1024 * es
        def mk(i, rows=rows, dtype=dtype):
            x = torch.randn(rows, 1024, generator=g).to(dtype).to(dev)
            r = torch.randn(rows, 1024, generator=g).to(dtype).to(dev)
            w = (1 + 0.02 * torch.randn(1024, generator=g)).to(dtype).to(dev)
            y, h = torch.empty_like(x), torch.empty_like(x)
            ours = lambda: K.fused_add_rms_norm(x, r, w, 1e-5, out=y, residual_out=h)  # noqa: E731
            def theirs():   # the eager add (optimized_decode.py:252), then the Triton norm
                torch.add(x, r, out=h)
                _triton_rms(ref, h, w, y, 1e-5)
            return ours, (theirs if tk else None)
        measure(f"add_rms_norm_{str(dtype)[6:]}_{rows}x1024", rot_sets(mk, nbytes), nbytes)
    # SiLU*mul (config 3)
    for t in (1, 64, 512, 4096, 32768):
        nbytes = t * 27648
        def mk(i, t=t):
            x = torch.randn(t, 9216, generator=g).to(torch.bfloat16).to(dev)
            y = torch.empty(t, 4608, dtype=torch.bfloat16, device=dev)
            return (lambda: K.fused_silu_mul(x, out=y)), ((lambda: _triton_silu(ref, x, y)) if tk else None)
        measure(f"silu_mul_bf16_T{t}", rot_sets(mk, nbytes), nbytes, launches=100 if t >= 32768 else 400)
    # RoPE + frame table + KV write (config 2 sweep, plus large-T points beyond it).
    # The reference has a one-token path only (triton_kernels.py:152-155), so its
    # column is at T = 1 (without a frame table, which it does not have).
    for t in (1, 64, 512, 4096, 16384, 32768):
        nbytes = t * BYTES_PER_TOKEN
        def mk(i, t=t):
            s = make_inputs(100 + i, t, dev)
            qo = torch.empty(1, t, HQ, D, dtype=torch.bfloat16, device=dev)
            theirs = None
            if t == 1:
                p = int(torch.randint(0, 2048, (1,), generator=g))
                s["pos"].fill_(p)
                s["slots"].fill_(p)
                if tk is not None:
                    rc = _ref_cache(ref, dev)
                    rc.set_write_position(p)
                    theirs = lambda: _ref_rope_kv_step(ref, s["q"], s["k"], s["v"], s["inv"], s["pos"], rc)  # noqa: E731
            return (lambda: launch(K, s, qo)), theirs
        measure(f"rope_kv_write_bf16_T{t}", rot_sets(mk, nbytes), nbytes, launches=100 if t >= 16384 else 400)
    nbytes = BYTES_PER_TOKEN - 128 + 256
    def mk_norm(i):
        s = make_inputs(200 + i, 1, dev)
        qw = (1 + 0.02 * torch.randn(D, generator=g)).to(torch.bfloat16).to(dev)
        kw = (1 + 0.02 * torch.randn(D, generator=g)).to(torch.bfloat16).to(dev)
        qo = torch.empty(1, 1, HQ, D, dtype=torch.bfloat16, device=dev)
        theirs = None
        if tk is not None:
            rc = _ref_cache(ref, dev)
            rc.set_write_position(int(s["slots"][0]))
            theirs = lambda: _ref_rope_kv_step(ref, s["q"], s["k"], s["v"], s["inv"], s["pos"], rc, qw, kw)  # noqa: E731
        return (lambda: K.fused_rope_kv_write(s["q"].view(1, 1, HQ, D), s["k"].view(1, 1, HK, D),
                                              s["v"].view(1, 1, HK, D), s["inv"], s["pos"], s["kc"], s["vc"],
                                              s["slots"], q_norm_w=qw, k_norm_w=kw, q_out=qo)), theirs
    measure("rope_kv_write_qknorm_decode_bf16", rot_sets(mk_norm, nbytes), nbytes)
    return out


# ------------------------------------------------------------ decode step

def _synthetic(dev, rank: int, batch: int, prompt: int):
    """The synthetic LFM2 (16 layers: 10 short-conv + 6 GQA 16/8/64, H 1024,
    FF 4608, vocab 80000, random bf16 weights std 0.02), `prompt` random ids and
    a 128-d speaker embedding per stream."""
    from kani_tts_b200.model import LFM2Config, synthetic_state_dict
    cfg = LFM2Config()
    sd = synthetic_state_dict(cfg, seed=0, device=dev)
    g = torch.Generator(device="cpu").manual_seed(1 + rank)
    ids = torch.randint(0, cfg.audio_tokens_start, (batch, prompt), generator=g).to(dev)
    spk = torch.randn(batch, cfg.speaker_emb_dim, generator=g).to(dev)
    return cfg, sd, ids, spk


def run_decode(dev, world, rank, batch: int, steps: int, prompt: int = 128) -> dict:
    """`prompt`-token prefill (plus the speaker embedding inserted at position 1),
    then `steps` greedy decode tokens per stream from a captured CUDA graph,
    static cache 2048 slots."""
    from kani_tts_b200.decode import DecodeEngine, FusedDecoder
    cfg, sd, ids, spk = _synthetic(dev, rank, batch, prompt)
    eng = DecodeEngine(FusedDecoder(cfg, sd, dev, batch=batch, max_len=2048))
    eng.start(ids, spk, steps + 8)
    eng.capture()
    eng.run(3)                                     # warm-up replays
    torch.cuda.synchronize(dev)
    _barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    eng.run(steps)
    e1.record()
    torch.cuda.synchronize(dev)
    _barrier(world)
    sec = _max_over_ranks(e0.elapsed_time(e1) / 1e3, world, dev)
    out = {"fused": {"us_per_step": round(sec / steps * 1e6, 2),
                     "tokens_per_s": round(world * batch * steps / sec, 1),
                     "kernel_flags": int(eng.dec.err_flag.item())}}
    del eng
    torch.cuda.empty_cache()
    out["config"] = (f"bs={batch} x {world} GPU(s), prompt {prompt}+speaker, {steps} decode steps, "
                     "S=2048, CUDA graph, greedy")
    return out


def run_decode_sampled(dev, world, rank, batch: int, steps: int, prompt: int = 128) -> dict:
    """Decode with the reference's sampling settings (temperature 0.5, top_p 0.85,
    repetition penalty 1.2, top-k 256; config.py:28-31), the sampler launched
    inside the captured step (no host work per token)."""
    from kani_tts_b200.decode import DecodeEngine, FusedDecoder
    from kani_tts_b200.sampling import SamplingParams
    cfg, sd, ids, spk = _synthetic(dev, rank, batch, prompt)
    sp = SamplingParams(seed=7 + rank)
    eng = DecodeEngine(FusedDecoder(cfg, sd, dev, batch=batch, max_len=2048), sampling=sp)
    eng.start(ids, spk, steps + 8)
    eng.capture()
    eng.run(3)
    torch.cuda.synchronize(dev)
    _barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    eng.run(steps)
    e1.record()
    torch.cuda.synchronize(dev)
    _barrier(world)
    sec = _max_over_ranks(e0.elapsed_time(e1) / 1e3, world, dev)
    audio = eng.dec.full_to_reduced[eng.generated[:, :steps]] >= 0
    out = {"fused_sampled": {"us_per_step": round(sec / steps * 1e6, 2),
                             "tokens_per_s": round(world * batch * steps / sec, 1),
                             "kernel_flags": int(eng.dec.err_flag.item()),
                             "tokens_in_reduced_vocab": bool(audio.all())}}
    del eng
    torch.cuda.empty_cache()
    out["config"] = (f"bs={batch} x {world} GPU(s), prompt {prompt}+speaker, {steps} decode steps, S=2048, "
                     f"sampling T={sp.temperature} top_p={sp.top_p} rp={sp.repetition_penalty} top_k={sp.top_k}")
    return out


def run_reference_decode(dev, ref, steps: int, prompt: int = 128, n_compare: int = 64) -> dict:
    """The reference's own decode engine at bs = 1 on the same synthetic model and
    GPU: ``OptimizedDecoder`` with its Triton kernels, captured into a CUDA graph
    by ``KaniInferenceEngine._initialize_cuda_graphs`` (inference_engine.py:
    230-331), then the loop body of ``generate`` (inference_engine.py:638-667)
    for `steps` tokens.

    The reference's HF prefill needs its full HF model class, so the prompt pass
    is this library's (``DecodeEngine.start``); its KV cache and conv states
    enter the reference engine through ``_initialize_cuda_graphs`` as the
    dynamic cache, as the reference's prefill results would.  Two loops:

    * ``reference_triton_graph`` (greedy): per token the loop's host writes
      (token, position, cache slot, mask slot), the graph replay, then
      ``reduced_to_full[argmax]`` on the device fed back as the next token
      — no host synchronisation, the step itself as the reference runs it.
      Before it, an untimed pass records the reference's first `n_compare`
      greedy tokens and logits; this library's decode step is then fed the
      same tokens from the same prefill state and its logits compared
      (``parity``).
    * ``reference_engine_sampled``: the same loop with the reference's
      ``_sample_next_token`` and its per-token ``.item()`` (sampling settings
      of config.py:28-31), the reference's serving loop.  It runs all `steps`
      tokens (an EOS does not stop the timing loop; ``eos_sampled`` counts
      them).

    Audio-count convention: the reference's graph loop starts after one HF
    decode step, so its index i is audio token i + 1 (position schedule
    inference_engine.py:615-619).  Here the first decode step is a graph step,
    so step k is audio token k: position = prefill length + (k // 4) * step."""
    import types as _t
    from baseline import reference as R
    from kani_tts_b200.decode import DecodeEngine, FusedDecoder
    cfg, sd, ids, spk = _synthetic(dev, 0, 1, prompt)
    mine = DecodeEngine(FusedDecoder(cfg, sd, dev, batch=1, max_len=2048))
    n_total = max(steps, n_compare) + 8   # the parity pass runs n_compare steps even for a short timing run
    mine.start(ids, spk, n_total)
    t_eff = prompt + 1
    dyn = _t.SimpleNamespace(
        key_cache=[mine.dec.k_cache[i][:, :, :t_eff].clone() if i in mine.dec.k_cache else torch.empty(0)
                   for i in range(cfg.num_hidden_layers)],
        value_cache=[mine.dec.v_cache[i][:, :, :t_eff].clone() if i in mine.dec.v_cache else torch.empty(0)
                     for i in range(cfg.num_hidden_layers)],
        conv_cache=[mine.dec.conv_state[i].clone() if i in mine.dec.conv_state else
                    torch.zeros(1, cfg.hidden_size, cfg.conv_L_cache, dtype=torch.bfloat16, device=dev)
                    for i in range(cfg.num_hidden_layers)])
    first = mine.input_ids.clone()
    mine.capture()
    mine.run(n_compare)
    torch.cuda.synchronize(dev)
    mine_tokens = mine.generated[0, :n_compare].clone()
    dec = mine.dec
    mine.graph = None

    math_sdp = torch.backends.cuda.math_sdp_enabled()   # the engine turns the math SDPA off
    model = R.stand_in_model(ref, cfg, sd, dev)
    eng = R.engine(ref, model, cfg, max_new_tokens=2048 - 512, temperature=0.5, top_p=0.85,
                   repetition_penalty=1.2)
    R.capture(eng, dyn, t_eff)
    od = eng.optimized_decoder
    sched = (t_eff + torch.arange(n_total, device=dev) // cfg.tokens_per_frame * cfg.audio_step).long()
    out = {}

    def body(i, next_token):
        # inference_engine.py:641-651 (the graph branch of the decode loop)
        eng.static_input_ids.copy_(next_token.view(1, 1))
        eng.static_position_ids[0, 0] = sched[i]
        step_offset = t_eff + i
        eng.static_cache_position[0] = step_offset
        eng.static_cache.set_write_position(step_offset)
        eng.static_mask[:, :, :, step_offset] = 0.0
        eng.cuda_graph.replay()
        eng.static_cache.advance_position()
        return eng.static_logits[:, -1, :]

    # parity pass (untimed): the reference's greedy tokens and logits; then this
    # library's decode step fed the same tokens from the same prefill state
    ref_logits, ref_inputs = [], [first.view(1, 1)]
    nt = first.view(1, 1)
    for i in range(n_compare):
        lg = body(i, nt)
        ref_logits.append(lg.clone())
        nt = od.reduced_to_full[lg.argmax(-1)].view(1, 1)
        ref_inputs.append(nt.clone())
    ref_tokens = torch.cat([t.view(-1) for t in ref_inputs[1:]])
    for i in dec.k_cache:
        dec.k_cache[i][:, :, :t_eff].copy_(dyn.key_cache[i])
        dec.v_cache[i][:, :, :t_eff].copy_(dyn.value_cache[i])
    for i in dec.conv_state:
        dec.conv_state[i].copy_(dyn.conv_cache[i])
    errs, coss, agree, clear, agree_clear = [], [], 0, 0, 0
    for i in range(n_compare):
        pos = sched[i:i + 1]
        slot = torch.tensor([t_eff + i], device=dev)
        mine_lg = dec.step_logits(ref_inputs[i], pos, slot, slot + 1)[:, -1, :].float()
        rl = ref_logits[i].float()
        errs.append(float((mine_lg - rl).abs().max() / rl.abs().max()))
        coss.append(float(torch.nn.functional.cosine_similarity(mine_lg.flatten(), rl.flatten(), dim=0)))
        same = int(mine_lg.argmax()) == int(rl.argmax())
        agree += same
        top2 = rl.flatten().topk(2).values
        if float(top2[0] - top2[1]) > 2.0 ** -5 * abs(float(top2[0])):
            clear += 1
            agree_clear += same
    same = (ref_tokens == mine_tokens).tolist()
    parity = {"steps": n_compare, "max_logit_err_frac": round(max(errs), 5), "min_cosine": round(min(coss), 6),
              "argmax_agree": f"{agree}/{n_compare}", "argmax_agree_where_clear": f"{agree_clear}/{clear}",
              "free_running_identical_prefix": same.index(False) if False in same else len(same),
              "how": "teacher-forced: this library's decode step fed the reference's greedy tokens from the "
                     "same prefill state; clear = top-2 margin above 2^-5 of the top logit"}
    eng._refresh_static_cache(dyn, t_eff)

    # greedy loop (timed)
    toks = torch.zeros(steps + 8, dtype=torch.long, device=dev)
    nt = first.view(1, 1)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for i in range(steps + 3):
        if i == 3:
            e0.record()
        nt = od.reduced_to_full[body(i, nt).argmax(-1)]
        toks[i] = nt.view(-1)[0]
    e1.record()
    torch.cuda.synchronize(dev)
    sec = e0.elapsed_time(e1) / 1e3
    out["reference_triton_graph"] = {
        "us_per_step": round(sec / steps * 1e6, 2), "tokens_per_s": round(steps / sec, 1),
        "path": "kani_tts OptimizedDecoder (Triton) captured by KaniInferenceEngine._initialize_cuda_graphs; "
                "generate() loop body with a device-side greedy choice"}
    out["parity"] = parity

    # the reference's serving loop: its sampler and .item() per token
    eng._refresh_static_cache(dyn, t_eff)
    gen = torch.zeros(1, prompt + steps + 16, dtype=torch.long, device=dev)
    gen[0, :prompt] = ids[0]
    gen_len = prompt
    gen[0, gen_len] = int(first.view(-1)[0])
    gen_len += 1
    nt = first.view(1, 1)
    eos = torch.tensor([cfg.eos_token_id], device=dev, dtype=torch.long)
    prev_is_eos, n_eos = None, 0
    for i in range(steps + 3):
        if i == 3:
            torch.cuda.synchronize(dev)
            e0.record()
        logits = body(i, nt)
        nt = eng._sample_next_token(logits, gen[:, :gen_len])          # :654
        tid = nt[0, 0].item()                                           # :655
        gen[0, gen_len] = tid
        gen_len += 1
        if prev_is_eos is not None and prev_is_eos.item():             # :661-667 (pipelined EOS check)
            n_eos += 1
        prev_is_eos = (nt.view(-1) == eos)
    e1.record()
    torch.cuda.synchronize(dev)
    sec_s = e0.elapsed_time(e1) / 1e3
    out["reference_engine_sampled"] = {
        "us_per_step": round(sec_s / steps * 1e6, 2), "tokens_per_s": round(steps / sec_s, 1),
        "eos_sampled": n_eos,
        "path": "generate() loop body: graph replay, _sample_next_token, .item() per token"}
    del eng, model, od, mine, dec
    torch.backends.cuda.enable_math_sdp(math_sdp)
    torch.cuda.empty_cache()
    out["config"] = (f"bs=1, prompt {prompt}+speaker (prefill by this library), {steps} decode steps, "
                     "static cache 2048 (max(prefill, 512) + 1536), reference sampling T=0.5 top_p=0.85 rp=1.2")
    return out


def run_gpu(args, world, rank, local):
    from kani_tts_b200 import _lib
    from kani_tts_b200 import fused_kernels as K
    _lib.load_library()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peak, peak_kind = _peaks()
    _lib.error_flag(dev)

    sets = [make_inputs(1000 * rank + i, device=dev) for i in range(N_SETS)]
    outs = [torch.empty(1, T_TOK, HQ, D, dtype=torch.bfloat16, device=dev) for _ in range(N_SETS)]
    fns = [lambda s=s, o=o: launch(K, s, o) for s, o in zip(sets, outs)]
    for i in range(max(3, args.warmup)):
        fns[i % N_SETS]()
    torch.cuda.synchronize(dev)

    c0 = _lib.launch_count()
    with ClockSampler(dev) as clocks:
        elapsed = time_graph_steps(fns, args.steps, dev, world)
    captured = _lib.launch_count() - c0        # launches recorded into the graphs
    elapsed_max = _max_over_ranks(elapsed, world, dev)
    per_rank_us = [round(s / args.steps * 1e6, 3) for s in _gather_over_ranks(elapsed, world, dev)]
    flags = _lib.read_and_clear_errors(dev)
    if flags:
        raise RuntimeError(f"kernel error flags set during the bench: {flags}")

    value = world * args.steps * STEP_BYTES / elapsed_max / 1e9
    per_launch_s = elapsed / args.steps
    achieved = STEP_BYTES / per_launch_s / 1e9

    extras = {}
    cpu = None
    _barrier(world)
    e = run_e2e(K, dev, min(args.steps, 200))
    e_max = _max_over_ranks(e["seconds"], world, dev)
    link = _max_over_ranks(host_link_copies(dev, e["h2d"], e["d2h"], e["steps"]), world, dev)
    e2e_line = {"value": round(world * e["steps"] * STEP_BYTES / e_max / 1e9, 3), "unit": UNIT,
                "h2d_bytes_per_step": e["h2d"], "d2h_bytes_per_step": e["d2h"], "steps": e["steps"],
                "ms_per_step": round(e_max / e["steps"] * 1e3, 4),
                "host_link_ceiling": {"value": round(world * e["steps"] * STEP_BYTES / link / 1e9, 3), "unit": UNIT,
                                      "ms_per_step": round(link / e["steps"] * 1e3, 4),
                                      "what": "the same copies per step with no kernel (slowest rank)"},
                "path": ("kani_tts_b200.fused_rope_kv_write (ctypes -> kani_rope_kv_write): one pinned "
                         "packed input buffer (Q|K|V rows, positions, slots) and one result buffer (rotated Q, "
                         "K and V caches) per step, copy-in / compute / copy-out streams over two buffer sets")}
    ref = None
    if not args.no_reference_gpu:
        from baseline import reference as R
        ref = R.import_reference() if R.available() else None
    if not args.no_decode:
        # decode steps: bs=1 and 64 streams per GPU, greedy and sampled
        extras["decode"] = {"bs1": run_decode(dev, world, rank, 1, args.decode_steps),
                            "bs64": run_decode(dev, world, rank, 64, args.decode_steps),
                            "bs1_sampled": run_decode_sampled(dev, world, rank, 1, args.decode_steps),
                            "bs64_sampled": run_decode_sampled(dev, world, rank, 64, args.decode_steps)}
        if rank == 0:
            # the reference's Triton + CUDA-graph engine on the same GPU (bs = 1)
            if ref is None:
                extras["decode"]["bs1_reference"] = {"unavailable": _ref_unavailable(args)}
            else:
                r = run_reference_decode(dev, ref, args.decode_steps)
                mine_g = extras["decode"]["bs1"]["fused"]["us_per_step"]
                mine_s = extras["decode"]["bs1_sampled"]["fused_sampled"]["us_per_step"]
                r["speedup_greedy"] = round(r["reference_triton_graph"]["us_per_step"] / mine_g, 3)
                r["speedup_sampled"] = round(r["reference_engine_sampled"]["us_per_step"] / mine_s, 3)
                extras["decode"]["bs1_reference"] = r
    copy_ref = None
    if rank == 0:
        copy_ref = same_traffic_copy(dev, STEP_BYTES // 2)
        if not args.no_sweep:
            extras["sweep"] = run_sweep(K, dev, peak, ref)
            if ref is None:
                extras["sweep"]["triton"] = {"unavailable": _ref_unavailable(args)}
        if world == 1 and not args.no_cpu:
            cpu = cpu_oracle_rate(args.cpu_seconds)
    if rank != 0:
        return
    traffic, traffic_src = _traffic_per_launch()
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": round(elapsed_max / args.steps * 1e3, 6),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) inputs, N(0,0.02) frame table)",
        "config": {"workload": WORKLOAD, "bytes_per_step": STEP_BYTES,
                   "l2": f"inputs rotated over {N_SETS} sets ({N_SETS * STEP_BYTES / 1e6:.0f} MB > 126 MB L2)",
                   "launch": "CUDA-graph replay of the kernel, one launch per step",
                   "parallelism": f"replicas x{world} (independent streams, no collectives)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind, "traffic": traffic,
                     "traffic_source": traffic_src,
                     "algorithmic_bytes": STEP_BYTES,
                     "kernel": "rope_bulk_kernel<bf16, NORM=0, TABLE=1, QI=2, KI=1, LOG2L=2>",
                     "same_traffic_copy": (None if copy_ref is None else
                                           {**copy_ref, "frac_of_it": round(achieved / copy_ref["GB_s"], 4)})},
        "e2e": e2e_line,
        "gpu_launches": args.steps,
        "graph_launches_captured": captured,
        "us_per_launch_by_rank": per_rank_us,
        "clocks": clocks.summary(),
    }
    if cpu is not None:
        line["cpu_baseline"] = {k: (round(v, 4) if isinstance(v, float) else v) for k, v in cpu.items()
                                if k in ("value", "unit", "cores", "kind", "sample")}
    line.update(extras)
    print(json.dumps(line), flush=True)


def same_traffic_copy(dev, nbytes: int, sets: int = 8, launches: int = 1000) -> dict:
    """A plain device copy of `nbytes` (the headline's read volume; the copy writes
    as much again), graph-replayed over rotating buffers like the headline: what
    the memory system gives a step of this size.  The measured peak comes from
    copies far larger, which amortise the start and the drain of each launch."""
    n = nbytes // 2
    srcs = [torch.randn(n, device=dev).to(torch.bfloat16) for _ in range(sets)]
    dsts = [torch.empty_like(x) for x in srcs]
    g = graph_of([lambda i=i: dsts[i % sets].copy_(srcs[i % sets]) for i in range(launches)])
    g.replay()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    g.replay()                           # lead-in, untimed
    e0.record()
    g.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    us = e0.elapsed_time(e1) * 1e3 / launches
    del g, srcs, dsts
    torch.cuda.empty_cache()
    return {"GB_s": round(2 * n * 2 / us / 1e3, 1), "us": round(us, 3), "bytes_read": 2 * n, "bytes_written": 2 * n}


def run_op(name: str, size: int, steps: int, warmup: int) -> dict:
    """Profiling aid: one fused op alone at one size, eager launches, seeded inputs."""
    from kani_tts_b200 import fused_kernels as K
    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(0)
    bf = torch.bfloat16

    def rn(*shape):
        return torch.randn(*shape, generator=g).to(bf).to(dev)
    if name == "silu_mul":
        x, y = rn(size, 9216), torch.empty(size, 4608, dtype=bf, device=dev)
        fn, nbytes = (lambda: K.fused_silu_mul(x, out=y)), size * 27648
    elif name == "add_rms_norm":
        x, r, w = rn(size, 1024), rn(size, 1024), rn(1024)
        o, h = torch.empty_like(x), torch.empty_like(x)
        fn, nbytes = (lambda: K.fused_add_rms_norm(x, r, w, 1e-5, out=o, residual_out=h)), size * 1024 * 8 + 2048
    elif name == "rope_kv_write":
        st = make_inputs(0, size, dev)
        qo = torch.empty(1, size, HQ, D, dtype=bf, device=dev)
        fn, nbytes = (lambda: launch(K, st, qo)), size * BYTES_PER_TOKEN
    elif name == "decode_attention":          # size = streams, 1629 valid slots of 2048
        q, kc, vc = rn(size, HQ, D), rn(size, HK, 2048, D), rn(size, HK, 2048, D)
        kv_len = torch.full((size,), 1629, dtype=torch.long, device=dev)
        out = torch.empty(size, HQ, D, dtype=bf, device=dev)
        fn, nbytes = (lambda: K.decode_attention(q, kc, vc, kv_len, out=out)), size * (2 * HK * 1629 * D * 2 + 2 * HQ * D * 2)
    elif name == "short_conv":               # size = streams, hidden 1024, L = 3
        bcx, stt, w = rn(size, 3 * 1024), rn(size, 1024, 3), rn(1024, 3)
        y = torch.empty(size, 1024, dtype=bf, device=dev)
        fn, nbytes = (lambda: K.short_conv_step(bcx, stt, w, out=y)), size * 1024 * 2 * (3 + 3 + 3 + 1) + 1024 * 6
    elif name == "sample":                   # size = streams, reduced vocab 15591, config sampling settings
        from kani_tts_b200 import sampling as KS
        v = 15591
        lg = rn(size, v)
        seen = KS.seen_bitmap(torch.randint(0, v, (size, 200), generator=g), v, device=dev)
        step = torch.zeros(1, dtype=torch.long, device=dev)
        tok = torch.empty(size, dtype=torch.long, device=dev)
        fn = (lambda: K.sample_tokens(lg, seen, temperature=0.5, top_p=0.85, repetition_penalty=1.2, seed=1,
                                      step=step, out=tok))
        nbytes = size * (v * 2 + seen.shape[1] * 4 + 8)
    elif name == "gemv_gate_up":               # size = streams; add + RMSNorm + gate/up GEMV + SiLU·mul
        from kani_tts_b200.fused_kernels import gemv
        x, r = rn(size, 1, 1024), rn(size, 1, 1024)
        nw, wt = rn(1024), rn(9216, 1024) * 0.03
        h, y = torch.empty_like(x), torch.empty(size, 1, 4608, dtype=bf, device=dev)
        fn = lambda: gemv(x, wt, norm_weight=nw, residual=r, residual_out=h, silu_pairs=True, out=y)  # noqa: E731
        nbytes = 9216 * 1024 * 2 + size * 1024 * 2 * 3 + size * 4608 * 2
    elif name in ("head_argmax", "head_tc", "head_cublas", "head_cublas_pad8"):
        rows, h = 15591, 1024                   # size = streams; reduced head 15591 x 1024
        hid, wt = rn(size, h), rn(rows, h) * 0.05
        imap = torch.arange(rows, device=dev) + 64410
        out = torch.empty(size, dtype=torch.long, device=dev)
        if name == "head_argmax":
            scratch = torch.zeros(size + 1, dtype=torch.long, device=dev)
            fn = lambda: K.head_argmax(hid, wt, imap, scratch=scratch, out=out)  # noqa: E731
        elif name == "head_tc":
            scratch = torch.zeros(size + 1, dtype=torch.int32, device=dev)
            fn = lambda: K.head_argmax_tc(hid, wt, imap, scratch=scratch, out=out)  # noqa: E731
        elif name == "head_cublas_pad8":        # head rows padded to a multiple of 8, logits sliced back
            wp = torch.zeros((rows + 7) // 8 * 8, h, dtype=bf, device=dev)
            wp[:rows].copy_(wt)
            fn = lambda: out.copy_(imap[torch.nn.functional.linear(hid, wp)[:, :rows].argmax(-1)])  # noqa: E731
        else:                                   # the reference's F.linear head + greedy argmax + map
            fn = lambda: out.copy_(imap[torch.nn.functional.linear(hid, wt).argmax(-1)])  # noqa: E731
        nbytes = rows * h * 2 + size * h * 2
    else:
        raise SystemExit(f"unknown op {name}")
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize(dev)
    us = e0.elapsed_time(e1) * 1e3 / steps
    # the same calls replayed from a CUDA graph: device time without the Python launch path
    per_graph = 50
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream(dev).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(per_graph):
            fn()
    graph.replay()
    torch.cuda.synchronize(dev)
    reps = max(1, steps // per_graph)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    us_g = e0.elapsed_time(e1) * 1e3 / (reps * per_graph)
    return {"op": name, "size": size, "us_per_call_eager": round(us, 3), "us_per_call_graph": round(us_g, 3),
            "bytes": nbytes, "GB_s": round(nbytes / us / 1e3, 1), "GB_s_graph": round(nbytes / us_g / 1e3, 1)}


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100000)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["kani_b200", "reference"], default="kani_b200")
    ap.add_argument("--no-sweep", action="store_true", help="skip the per-op sweep")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode-step measurements")
    ap.add_argument("--no-reference-gpu", action="store_true",
                    help="skip the reference's Triton kernels and Triton + CUDA-graph engine on the GPU")
    ap.add_argument("--decode-steps", type=int, default=1500)
    ap.add_argument("--decode-only", action="store_true", help="profiling aid: run only the decode arms")
    ap.add_argument("--decode-batch", type=int, default=1, help="streams for --decode-only")
    ap.add_argument("--op", default=None, help="profiling aid: run one fused op alone "
                    "(silu_mul, add_rms_norm, rope_kv_write, decode_attention, short_conv, sample, "
                    "head_argmax, head_tc, head_cublas, head_cublas_pad8, gemv_gate_up)")
    ap.add_argument("--size", type=int, default=4096, help="rows / tokens / streams for --op")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.op:
        print(json.dumps(run_op(args.op, args.size, args.steps, args.warmup)), flush=True)
        return
    if args.decode_only:
        # profiling aid: only the bs=1 decode arms, one JSON line with the decode results
        world, rank, local = _dist_init()
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        res = run_decode(dev, world, rank, args.decode_batch, args.decode_steps)
        res_s = run_decode_sampled(dev, world, rank, args.decode_batch, args.decode_steps)
        if rank == 0 and args.decode_batch == 1 and not args.no_reference_gpu:
            from baseline import reference as R
            if R.available():
                res["reference"] = run_reference_decode(dev, R.import_reference(), args.decode_steps)
        if rank == 0:
            print(json.dumps({"decode": res, "decode_sampled": res_s}), flush=True)
        return
    if args.impl == "reference":
        # CPU arm: rank 0 alone measures; other ranks exit without work or a process group
        run_reference(args, int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")))
        return
    world, rank, local = _dist_init()
    try:
        run_gpu(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
