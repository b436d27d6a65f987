"""Benchmark of the B200 decode sparse-attention path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (config 2): batched decode, attention path only, all 43 layers;
64 sequences per GPU at 32768 raw-token context (8192 compressed entries),
indexer top-2048 plus a 128-token window, every layer with its own seeded
caches, indexer weights and sinks.  One "step" = one decode step of all 43
layers (act_quant + window write, indexer compressor, indexer score, top-k,
attention compressor, sparse attention) for the 64 sequences, positions
advancing on the device.  Inputs are synthetic (seeded ~N(0,1), indexer
weights ~N(0,0.02)); the 29 GB of caches per GPU are far larger than L2, so
no L2 flush is needed between steps.

Multi-GPU (torchrun): batch split with no collective on the path - each rank
runs its own 64 sequences ("scaling": "weak"); the step time is the max over
ranks of the CUDA-event time.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "tt-deepseek-v4_b200"))
sys.path.insert(0, ROOT)

METRIC = "sparse-attn decode µs/layer & tok/s; HBM GB/s % of peak at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=43)
    ap.add_argument("--batch", type=int, default=64, help="sequences per GPU")
    ap.add_argument("--ctx", type=int, default=32768)
    ap.add_argument("--topk", type=int, default=2048)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-seq-split", action="store_true",
                    help="skip the config-3 sequence-split record that the default (cfg2) run adds")
    ap.add_argument("--no-projections", action="store_true",
                    help="skip the record of the projections around the path that the default (cfg2) run adds")
    ap.add_argument("--breakdown", action="store_true", help="print per-kernel timings to stderr")
    ap.add_argument("--workload", choices=["cfg0", "cfg1", "cfg2", "cfg3", "cfg4"], default="cfg2",
                    help="cfg0: one layer, batch 1, 4096-token context; cfg1: compressor emit path alone; "
                         "cfg2: batched decode, batch split; cfg3: one 256k context, sequence split; "
                         "cfg4: 4096-token prefill chunk")
    ap.add_argument("--comm", choices=["p2p", "nccl"], default="p2p",
                    help="cfg3 exchanges: peer-memory stores over NVLink, or NCCL all-gathers")
    a = ap.parse_args()
    if a.workload == "cfg3" and "--ctx" not in sys.argv:
        a.ctx = 262144
    if a.workload == "cfg0":
        # 43 independent single-layer problems per step, so the timed working set exceeds L2
        for flag, attr, val in (("--batch", "batch", 1), ("--ctx", "ctx", 4096), ("--topk", "topk", 512),
                                ("--layers", "layers", 43)):
            if flag not in sys.argv:
                setattr(a, attr, val)
    return a


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def read_traffic():
    """Per-launch DRAM traffic of each kernel from the committed ncu summary
    (profiles/roofline_traffic.txt: `kernel workload bytes_per_launch`)."""
    out = {}
    p = os.path.join(ROOT, "profiles", "roofline_traffic.txt")
    if os.path.exists(p):
        for line in open(p):
            parts = line.split()
            if len(parts) >= 3 and not line.startswith("#"):
                try:
                    out[(parts[0], parts[1])] = float(parts[2])
                except ValueError:
                    pass
    return out


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ workload

def algorithmic_bytes(B, t_active, k, W, H=64, D=512, Hi=64, Di=128):
    """Bytes the algorithm must move per layer-step for B sequences (gathered
    rows, not the full cache), per kernel."""
    K = W + k
    attn = B * (K * D * 2 + H * D * 2 * 2 + K * 4)          # gather + q + o + indices
    idx = B * (t_active * Di * 2 + Hi * Di * 2 + Hi * 4 + t_active * 4)  # keys + q + w + scores
    topk = B * (t_active * 4 + k * 4)
    cmp = B * (2 * (2 * D) * 2 + 2 * (2 * Di) * 2 + (2 * 8 * 2 * D * 4) // 4 + (2 * 8 * 2 * Di * 4) // 4 + 2 * D)
    kvw = B * (D * 2 * 2)
    return {"sparse_attn": attn, "indexer_score": idx, "indexer_topk": topk, "compressor": cmp,
            "kv_window_write": kvw}


def build_path(args, dev, seed):
    import torch
    from dsv4attn.layer import DecodeLayer, DecodePath, LayerInputs
    from dsv4attn.tables import PathArgs
    pa = PathArgs(index_topk=args.topk)
    max_seq = args.ctx + 4096
    g = torch.Generator(device=dev).manual_seed(seed)
    layers = []
    for li in range(args.layers):
        L = DecodeLayer(pa, args.batch, max_seq, dev)
        L.kv_cache.normal_(generator=g)
        L.idx_cache.normal_(generator=g)
        L.cmp_kv.normal_(generator=g)
        L.cmp_sc.normal_(generator=g)
        L.icmp_kv.normal_(generator=g)
        L.icmp_sc.normal_(generator=g)
        L.ape.normal_(generator=g)
        L.iape.normal_(generator=g)
        L.gamma.normal_(generator=g).mul_(0.02).add_(1.0)
        L.igamma.normal_(generator=g).mul_(0.02).add_(1.0)
        L.sink.normal_(generator=g)
        layers.append(L)
    path = DecodePath(layers, max_seq)
    inputs = []
    for li in range(args.layers):
        x = LayerInputs.empty(pa, args.batch, dev)
        for t in x.tensors():
            t.normal_(generator=g)
        x.iw.mul_(0.02)
        inputs.append(x)
    outs = [torch.empty(args.batch, 64, 512, dtype=torch.bfloat16, device=dev) for _ in range(args.layers)]
    return pa, path, inputs, outs


def time_kernels(path, inputs, outs, reps=3):
    """Device time per launch of each kernel kind: the op is captured over all
    layers (distinct caches, so nothing stays in L2) in one CUDA graph and the
    graph is timed with CUDA events on the replaying stream, so host launch
    overhead does not enter the figure."""
    import torch
    from dsv4attn import ops
    res = {}

    def run(name, fn):
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            fn()
        torch.cuda.current_stream().wait_stream(st)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        g.replay()
        torch.cuda.synchronize()
        cur = torch.cuda.current_stream()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        best = None
        for _ in range(reps):
            e0.record(cur)
            g.replay()
            e1.record(cur)
            e1.synchronize()
            ms = e0.elapsed_time(e1) / len(path.layers)
            best = ms if best is None else min(best, ms)
        res[name] = best
        del g

    run("sparse_attn", lambda: [ops.sparse_attn(x.q, L.kv_cache, L.idx, L.sink, path.scale, out=o, ws=L.ws,
                                                lead_cols=L.win, lead_ready=True)
                                for L, x, o in zip(path.layers, inputs, outs)])
    run("indexer_score", lambda: [ops.indexer_score(x.iq, L.idx_cache, x.iw, L.T_max, out=L.score,
                                                    t_valid=path.t_active) for L, x in zip(path.layers, inputs)])
    run("indexer_topk", lambda: [ops.indexer_topk(L.score, path.t_active, L.k, L.win, T=L.T_max, mask_mode=1,
                                                  out=L.idx[:, L.win:], ws=L.ws) for L in path.layers])
    # the layer's small stages in one launch (the step runs it beside the
    # indexer score; timed alone here)
    a = path.args
    run("layer_prologue", lambda: [ops.layer_prologue(
        (x.icmp_kv, x.icmp_score, L.iape, L.icmp_kv, L.icmp_sc, L.igamma, L.idx_cache),
        (x.cmp_kv, x.cmp_score, L.ape, L.cmp_kv, L.cmp_sc, L.gamma, L.kv_cache), path.cos, path.sin, path.pos,
        path.t_active, x.iq, x.iw, L.score, L.T_max, x.kv, L.idx, L.win, L.ratio, eps=a.norm_eps,
        rope_dim=a.rope_head_dim) for L, x in zip(path.layers, inputs)])
    return res


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def _oracle_state(O, torch, B, W, T, k, ctx, g):
    cos, sin = O.rope_tables(64, ctx + 8, compressed=True)
    ckv, csc = O.compressor_init_state(B, 512, 4, True)
    ikv, isc = O.compressor_init_state(B, 128, 4, True)
    return O.LayerState(kv_cache=torch.randn(B, W + T + 4, 512, generator=g).to(torch.bfloat16),
                        idx_kv_cache=torch.randn(B, T + 4, 128, generator=g).to(torch.bfloat16),
                        cmp_kv=ckv.normal_(generator=g), cmp_sc=csc.normal_(generator=g),
                        icmp_kv=ikv.normal_(generator=g), icmp_sc=isc.normal_(generator=g),
                        ape=torch.randn(4, 1024, generator=g), gamma=torch.ones(512),
                        iape=torch.randn(4, 256, generator=g), igamma=torch.ones(128),
                        sink=torch.randn(64, generator=g), cos=cos, sin=sin, win=W, ratio=4, index_topk=k,
                        scale=512 ** -0.5)


def _oracle_inputs(torch, B, g):
    bf = torch.bfloat16
    return [torch.randn(B, 1, 64, 512, generator=g).to(bf), torch.randn(B, 512, generator=g).to(bf),
            torch.randn(B, 1024, generator=g), torch.randn(B, 1024, generator=g),
            torch.randn(B, 64, 128, generator=g).to(bf), torch.randn(B, 256, generator=g),
            torch.randn(B, 256, generator=g), 0.02 * torch.randn(B, 64, generator=g)]


def cpu_baseline_sample(args, seconds=12.0, n_seq=None):
    """Time the CPU oracle (all host threads) on a bounded sample of the same
    decode workload: ``n_seq`` sequences (default min(2, batch)) of one layer
    at the run's shapes (context, top-k, window 128); report tok/s for the
    ``args.layers``-layer step."""
    import torch
    import oracle as O
    torch.set_num_threads(host_cores())
    g = torch.Generator().manual_seed(0)
    W, k, ctx = 128, args.topk, args.ctx
    T = ctx // 4
    B = n_seq if n_seq is not None else min(2, args.batch)
    st = _oracle_state(O, torch, B, W, T, k, ctx, g)
    x = _oracle_inputs(torch, B, g)
    pos = ctx - 1          # every repetition is the same decode step (state rewritten in place)
    n = 0
    t0 = time.perf_counter()
    while True:
        O.decode_layer_step(st, pos, *x)
        n += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = (time.perf_counter() - t0) / n          # seconds per layer-step of B sequences
    tok_s = B / (dt * args.layers)
    return {"value": tok_s, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{n} decode steps of 1 layer x {B} sequence(s) at ctx {ctx} (T={T}, k={k}, W=128), "
                      f"{dt * 1e3:.1f} ms per layer-step, scaled to {args.layers} layers"}


def cpu_baseline_cfg1(seconds=10.0):
    """CPU oracle of config 1: the compressor emit path, batch 32, d 512,
    ratio 4, non-overlap state; timed over consecutive steps from position 0."""
    import torch
    import oracle as O
    torch.set_num_threads(host_cores())
    g = torch.Generator().manual_seed(11)
    B, d, r = 32, 512, 4
    kv_row = torch.randn(B, d, generator=g).to(torch.bfloat16).float()
    sc_row = torch.randn(B, d, generator=g).to(torch.bfloat16).float()
    ape = 0.1 * torch.randn(r, d, generator=g)
    gamma = 1 + 0.02 * torch.randn(d, generator=g)
    cos, sin = O.rope_tables(64, 1100, compressed=True)
    kvs, scs = O.compressor_init_state(B, d, r, False)
    cache = torch.zeros(B, 1000 // r + 2, d, dtype=torch.bfloat16)
    n = 0
    t0 = time.perf_counter()
    while n < 1000:
        O.compressor_step(kvs, scs, kv_row, sc_row, ape, gamma, cos, sin, n, r, False, kv_cache=cache)
        n += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = (time.perf_counter() - t0) / n
    return {"value": B / dt, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{n} compressor steps from position 0 (batch {B}, d {d}, ratio {r}), {dt * 1e6:.1f} us per step"}


def cpu_baseline_cfg4(seconds=10.0, group=4):
    """CPU oracle of config 4 on a slice of the prefill chunk: groups of
    ``group`` tokens from the end of the 4096-token chunk (the oracle gathers
    a copy of the keys per token, so a group stays small), each against the
    full 32768-entry key set with per-token top-2048 + causal window, until
    ``seconds`` have passed; reported as tok/s of that slice."""
    import torch
    import oracle as O
    torch.set_num_threads(host_cores())
    g = torch.Generator().manual_seed(77)
    S, T, n_hist, k, W = 4096, 32768, 127, 2048, 128
    base = 131072 - S
    n_raw = n_hist + S
    kv = torch.randn(n_raw + T, 512, generator=g).to(torch.bfloat16)
    ikeys = torch.randn(T, 128, generator=g).to(torch.bfloat16)
    sink = torch.randn(64, generator=g)
    n_tok = 0
    t0 = time.perf_counter()
    while n_tok < S:
        rows = list(range(S - n_tok - group, S - n_tok))
        q = torch.randn(group, 64, 512, generator=g).to(torch.bfloat16)
        iq = torch.randn(group, 64, 128, generator=g).to(torch.bfloat16)
        iw = 0.02 * torch.randn(group, 64, generator=g)
        O.prefill_chunk(q, kv, n_raw, iq, ikeys, iw, sink, base, n_hist, T, k, W=W, rows=rows)
        n_tok += group
        if time.perf_counter() - t0 > seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": n_tok / dt, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"the last {n_tok} of the chunk's {S} tokens in groups of {group} (T={T}, top-{k}, "
                      f"window {W}), {dt:.1f} s"}


def run_reference(args, rank, world):
    """--impl reference: the reference's own CPU path is not runnable here (it
    needs ttnn/tt-lang on Tenstorrent hardware), so the oracle port stands in,
    timed on the host cores; rank 0 only."""
    if rank != 0:
        return
    cb = cpu_baseline_sample(args, seconds=max(8.0, 2.0 * args.steps))
    line = {"metric": METRIC, "impl": "reference", "value": cb["value"], "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": args.batch * 1e3 / cb["value"] if cb["value"] else None,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) caches, indexer weights N(0,0.02))",
            "config": {"workload": "cfg2 batched decode, 43 layers, 64 seq/GPU, ctx 32768, top-2048 + window 128",
                       "global_batch": args.batch * world, "seq_len": args.ctx, "parallelism": f"dp{world}"},
            "cpu_baseline": cb,
            "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def log(msg: str) -> None:
    print(f"[bench {time.strftime('%H:%M:%S')}] {msg}", file=sys.stderr, flush=True)


def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    import torch
    import torch.distributed as dist
    from dsv4attn import ops

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    if args.workload == "cfg3":
        run_cfg3(args, rank, world, dev)
        return
    if args.workload == "cfg4":
        run_cfg4(args, rank, world, dev)
        return
    if args.workload == "cfg1":
        run_cfg1(args, rank, world, dev)
        return

    log("building layers")
    pa, path, inputs, outs = build_path(args, dev, seed=1234 + rank)
    path.set_positions(args.ctx - 1)
    torch.cuda.synchronize()
    log("capturing the step graph")
    graph = path.capture(inputs, outs, warmup=1)
    path.set_positions(args.ctx - 1)
    torch.cuda.synchronize()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    ops.raise_for_status(path.status, "warm-up steps")
    log("warm-up done; timing")
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0.record(st)
    for _ in range(args.steps):
        graph.replay()
    e1.record(st)
    torch.cuda.synchronize()
    ms_total = e0.elapsed_time(e1)
    # per-replay times (separate loop, events around every replay) for median / min
    per = []
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]
    for i in range(args.steps):
        ev[2 * i].record(st)
        graph.replay()
        ev[2 * i + 1].record(st)
    torch.cuda.synchronize()
    per = sorted(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(args.steps))
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    if world > 1:
        t = torch.tensor([ms_total, per[len(per) // 2], per[0]], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t[0].item())
        per_med, per_min = float(t[1].item()), float(t[2].item())
    else:
        per_med, per_min = per[len(per) // 2], per[0]
    ops.raise_for_status(path.status, "timed steps")
    ms_step = ms_total / args.steps
    tok_s = world * args.batch * args.steps / (ms_total / 1e3)
    us_layer = ms_step * 1e3 / args.layers

    t_active = (args.ctx + args.warmup + args.steps) // 4
    ab = algorithmic_bytes(args.batch, t_active, args.topk, 128)
    bytes_step = sum(ab.values()) * args.layers
    hbm, hbm_kind = peaks()

    # per-kernel CUDA-event timings -> dominant kernel roofline
    log(f"timed: {ms_step:.3f} ms/step; per-kernel timings")
    kt = time_kernels(path, inputs, outs)
    # the dominant kernel among those the workload's byte count covers (the
    # layer prologue is latency-bound, with no roofline of its own)
    dom = max((k for k in kt if k in ab), key=kt.get)
    achieved = ab[dom] / (kt[dom] * 1e-3) / 1e9
    # ncu DRAM bytes of this workload's dominant kernel (None where no capture
    # of that workload is committed)
    traffic = read_traffic().get((dom, args.workload))
    roofline = {"bound": "hbm", "kernel": dom, "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                "frac": round(achieved / hbm, 4), "traffic": traffic,
                "peak_kind": f"{hbm_kind} (MEASURED_PEAKS.json hbm_gbs)" if hbm_kind == "measured" else "fallback",
                "algorithmic_bytes_per_launch": ab[dom], "us_per_launch": round(kt[dom] * 1e3, 2),
                "kernels_us": {k: round(v * 1e3, 2) for k, v in kt.items()}}
    step_gbs = bytes_step / (ms_step * 1e-3) / 1e9

    e2e = None
    if not args.no_e2e:
        log("end-to-end (host buffers)")
        e2e = measure_e2e(args, path, inputs, outs, dev, world)

    seq_split = None
    if args.workload == "cfg2" and not args.no_seq_split:
        log("config-3 sequence split record")
        seq_split = seq_split_record(args, rank, world, dev)

    projections = None
    if args.workload == "cfg2" and rank == 0 and not args.no_projections:
        log("projections record")
        projections = projections_record(args, dev)

    line = None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(tok_s, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "us_per_layer": round(us_layer, 2),
            "ms_per_step_median": round(per_med, 4), "ms_per_step_min": round(per_min, 4),
            "step_hbm_gbs": round(step_gbs, 1), "step_hbm_frac": round(step_gbs / hbm, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) caches/inputs, indexer weights N(0,0.02), random-init layer params)",
            "config": {"workload": (f"cfg2 batched decode: {args.layers} layers, {args.batch} seq/GPU, ctx {args.ctx} "
                                    f"({args.ctx // 4} compressed), indexer top-{args.topk} + window 128, "
                                    "H=64 D=512, Hi=64 Di=128") if args.workload == "cfg2" else
                                   (f"cfg0 single-layer decode step: batch {args.batch}, ctx {args.ctx} "
                                    f"({args.ctx // 4} compressed), top-{args.topk} + window 128"),
                       "global_batch": args.batch * world, "seq_len": args.ctx, "layers": args.layers,
                       "parallelism": f"dp{world} (batch split, no collective)",
                       "l2": f"working set {sum(L.nbytes() for L in path.layers) / 1e9:.2f} GB/GPU vs 126 MB L2; "
                             "no flush between steps (each layer's caches are read once per step)"},
            "roofline": roofline, "clocks": clk, "gpu_launches": path.launches_per_step() * args.steps,
        }
        if e2e is not None:
            line["e2e"] = e2e
        if seq_split is not None:
            line["seq_split"] = seq_split
        if projections is not None:
            line["projections"] = projections
    if rank == 0 and world == 1 and not args.no_cpu:
        log("CPU baseline sample")
        line["cpu_baseline"] = cpu_baseline_sample(args)
    if world > 1:
        dist.barrier()
        path.graph = None
        del graph
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def cfg3_build(args, rank, world, dev, p2p: bool):
    """One long context (args.ctx tokens, args.ctx / 4 compressed entries),
    its compressed KV and indexer keys split contiguously over ``world``
    ranks; returns (shard, path, inputs, outs, comm)."""
    import torch
    from dsv4attn.dist import P2PComm, SeqShard, SeqSplitPath, TorchDistComm
    from dsv4attn.layer import LayerInputs
    from dsv4attn.tables import PathArgs
    pa = PathArgs(index_topk=args.topk)
    T_total = args.ctx // 4
    max_seq = args.ctx + 4096
    shard = SeqShard(pa, 1, T_total, rank, world, dev, k=args.topk, n_layers=args.layers, max_seq_len=max_seq,
                     peer_exchange=p2p and world > 1)
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    for L in shard.layers:
        L.kv.normal_(generator=g)
        L.keys.normal_(generator=g)
        for t in (L.cmp_kv, L.cmp_sc, L.icmp_kv, L.icmp_sc, L.ape, L.iape):
            t.normal_(generator=g)
    gi = torch.Generator(device=dev).manual_seed(99)   # replicated inputs: same seed on every rank
    for L in shard.layers:
        L.sink.normal_(generator=gi)
    inputs = []
    for _ in range(args.layers):
        x = LayerInputs.empty(pa, 1, dev)
        for t in x.tensors():
            t.normal_(generator=gi)
        x.iw.mul_(0.02)
        inputs.append(x)
    outs = [torch.empty(1, 64, 512, dtype=torch.bfloat16, device=dev) for _ in range(args.layers)]
    comm = (P2PComm(shard) if p2p else TorchDistComm()) if world > 1 else None
    return shard, SeqSplitPath(shard, comm), inputs, outs, comm


def cfg3_measure(args, rank, world, dev, p2p: bool = True, sample_clocks: bool = True):
    """Time config 3 (sequence split over ``world`` ranks; every rank of the
    default process group takes part when world > 1) as a CUDA graph of all
    layers; returns {ms_step, us_per_layer, tok_s, timing, clocks}."""
    import torch
    import torch.distributed as dist
    from dsv4attn import ops
    shard, path, inputs, outs, comm = cfg3_build(args, rank, world, dev, p2p)
    shard.set_positions(args.ctx - 1)
    torch.cuda.synchronize()
    path.step(inputs, outs)                    # eager warm-up (also sizes the workspace)
    torch.cuda.synchronize()
    graph, mode = None, "graph"
    try:
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            path.step(inputs, outs)
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            path.step(inputs, outs)
    except Exception as e:                     # capture of the collectives refused: time eagerly
        log(f"cfg3 graph capture failed ({type(e).__name__}: {e}); timing eagerly")
        graph, mode = None, "eager"
        torch.cuda.synchronize()
    shard.set_positions(args.ctx - 1)
    torch.cuda.synchronize()

    def one():
        if graph is not None:
            graph.replay()
        else:
            path.step(inputs, outs)

    for _ in range(args.warmup):
        one()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(int(str(dev).split(":")[-1])) if sample_clocks else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0.record(st)
    for _ in range(args.steps):
        one()
    e1.record(st)
    torch.cuda.synchronize()
    ms_total = e0.elapsed_time(e1)
    clk = clocks.stop() if clocks else None
    if world > 1:
        t = torch.tensor([ms_total], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    ops.raise_for_status(shard.status, "cfg3 steps")
    ms_step = ms_total / args.steps
    if world > 1:
        dist.barrier()
    del graph
    torch.cuda.synchronize()
    if comm is not None:
        if world > 1:
            dist.barrier()
        comm.close()
    return {"ms_step": ms_step, "us_per_layer": ms_step * 1e3 / args.layers, "tok_s": 1e3 / ms_step,
            "timing": mode, "clocks": clk}


def cfg3_cpu_baseline(args, seconds=12.0):
    """CPU oracle of config 3: one decode step of one layer of the single
    long context (all compressed entries, no split), scaled to args.layers."""
    return cpu_baseline_sample(args, seconds=seconds, n_seq=1)


def run_cfg3(args, rank, world, dev):
    """Config 3: batch 1, one context of args.ctx tokens (args.ctx / 4
    compressed entries), compressed KV and indexer keys split contiguously
    over the ranks; per layer two exchanges (candidates, partials) over
    NVLink peer memory (--comm p2p) or NCCL all-gathers.  All 43 layers with
    their own shards; one step = one decode step of all layers.  "scaling":
    "strong" (the context is fixed as N grows)."""
    import torch.distributed as dist
    T_total = args.ctx // 4
    p2p = args.comm == "p2p"
    log(f"cfg3: building {args.layers} sharded layers (T={T_total}, rank {rank}/{world})")
    r = cfg3_measure(args, rank, world, dev, p2p=p2p)
    W, k, D, Di = 128, args.topk, 512, 128
    per_layer = T_total * Di * 2 + (W + k) * D * 2 + 64 * D * 2 * 2 + 64 * Di * 2 + 2 * T_total * 4
    hbm, hbm_kind = peaks()
    gbs = per_layer / (r["us_per_layer"] * 1e-6) / 1e9
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(r["tok_s"], 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(r["ms_step"], 4),
            "us_per_layer": round(r["us_per_layer"], 2), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) shards/inputs, indexer weights N(0,0.02))",
            "config": {"workload": f"cfg3 long-context decode: batch 1, ctx {args.ctx} ({T_total} compressed), "
                                   f"top-{k} + window {W}, {args.layers} layers, sequence split over {world} GPU(s)",
                       "global_batch": 1, "seq_len": args.ctx, "layers": args.layers,
                       "parallelism": f"sequence split x{world} ("
                                      + ("peer-memory exchange over NVLink" if p2p else
                                         ("NCCL all-gather" if world > 1 else "no exchange")) + ")",
                       "timing": r["timing"]},
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm * world, "unit": "GB/s",
                         "frac": round(gbs / (hbm * world), 4), "traffic": None,
                         "peak_kind": f"{hbm_kind} x {world} GPUs",
                         "algorithmic_bytes_per_layer": per_layer},
            "clocks": r["clocks"],
        }
        if world == 1 and not args.no_cpu:
            log("CPU baseline sample")
            line["cpu_baseline"] = cfg3_cpu_baseline(args)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def seq_split_record(args, rank, world, dev):
    """Config 3 beside the default run (the sequence split the scaling target
    is set on): the N-way split over every rank, and on rank 0 alone the
    1-GPU step it is compared with.  Returns the sub-object for rank 0's line
    (None elsewhere)."""
    import copy
    import torch
    import torch.distributed as dist
    a3 = copy.copy(args)
    a3.ctx, a3.topk, a3.layers = 262144, 2048, args.layers
    a3.steps, a3.warmup = max(10, args.steps), max(3, args.warmup)
    one = None
    if world > 1:
        dist.barrier()
    if rank == 0:
        one = cfg3_measure(a3, 0, 1, dev, p2p=False, sample_clocks=False)
        torch.cuda.empty_cache()
    if world > 1:
        dist.barrier()
        split = cfg3_measure(a3, rank, world, dev, p2p=True, sample_clocks=False)
        torch.cuda.empty_cache()
    else:
        split = one
    if rank != 0:
        return None
    return {"workload": f"cfg3 long-context decode: batch 1, ctx {a3.ctx} ({a3.ctx // 4} compressed), "
                        f"top-{a3.topk} + window 128, {a3.layers} layers, sequence split",
            "n_gpus": world, "us_per_layer": round(split["us_per_layer"], 2), "tok_s": round(split["tok_s"], 2),
            "us_per_layer_1gpu": round(one["us_per_layer"], 2), "tok_s_1gpu": round(one["tok_s"], 2),
            "exchange": "peer-memory stores over NVLink" if world > 1 else "none",
            "scaling": "strong", "timing": split["timing"]}


# the per-layer decode projections at DeepSeek-V4-Flash dims (dim 4096, q_lora
# 1024, 64 x 512 heads, 8 wo_a groups of o_lora 1024, indexer 64 x 128):
# (name, output rows over all groups, K per group, groups)
PROJECTIONS = (("wq_a", 1024, 4096, 1), ("wq_b", 32768, 1024, 1), ("wkv", 512, 4096, 1),
               ("compressor wkv|wgate", 2048, 4096, 1), ("indexer compressor wkv|wgate", 512, 4096, 1),
               ("indexer wq_b + q rotary", 8192, 1024, 1), ("weights_proj", 64, 4096, 1),
               ("wo_a (8 groups)", 8192, 4096, 8), ("wo_b", 4096, 8192, 1))
# the launches DeviceAttention runs them as: the projections of x in one
# weight, those of q_lora in another (the indexer's q rotary on its columns),
# then wo_a and wo_b: (name, rows, K, groups, rotary start column or None)
PROJECTION_LAUNCHES = (("x: wq_a|wkv|compressor wkv|wgate|indexer compressor wkv|wgate|weights_proj",
                        1024 + 512 + 2048 + 512 + 64, 4096, 1, None),
                       ("q_lora: wq_b|indexer wq_b + q rotary", 32768 + 8192, 1024, 1, 32768),
                       ("wo_a (8 groups)", 8192, 4096, 8, None), ("wo_b", 4096, 8192, 1, None))


def projections_record(args, dev, reps=10, copies=4):
    """The projections either side of the path (the step before it and the
    one after) through dsa_linear at config-2's batch, in the launches the
    block runs them as (PROJECTION_LAUNCHES: the projections sharing an
    input stored as one weight).  `copies` layers' worth with their own
    weights (so nothing is re-read from L2) run back to back from one CUDA
    graph; the time per layer is the graph's CUDA-event time over `copies`,
    median of `reps`.  cuBLAS (torch.matmul / bmm) on the same operands is
    the library reference point, both as the reference's nine matmuls and
    as the same four merged ones."""
    import torch
    from dsv4attn import ops
    B = args.batch
    hbm, _ = peaks()
    g = torch.Generator(device=dev).manual_seed(99)
    st = torch.cuda.current_stream()
    cos = torch.rand(args.ctx + 8, 32, device=dev, generator=g)
    sin = torch.rand(args.ctx + 8, 32, device=dev, generator=g)
    pos = torch.full((B,), args.ctx - 1, dtype=torch.int32, device=dev)

    def operands(table):
        layers = []
        for _ in range(copies):
            ents = []
            for ent in table:
                name, NT, K, G = ent[:4]
                col0 = ent[4] if len(ent) > 4 else None
                w = (torch.randn(NT, K, device=dev, generator=g) * K ** -0.5).to(torch.bfloat16)
                x = torch.randn(B, G * K, device=dev, generator=g).to(torch.bfloat16)
                y = torch.empty(B, NT, dtype=torch.bfloat16, device=dev)
                rope = (cos, sin, pos, 128, 64, col0) if col0 is not None else None
                ents.append((name, NT, K, G, w, ops.pack_linear_weight(w, groups=G), x, y, rope))
            layers.append(ents)
        return layers

    def native(layers, only=None):
        for ents in layers:
            for name, NT, K, G, w, wp, x, y, rope in ents:
                if only is None or name == only:
                    ops.linear(x, wp, out=y, rope=rope)

    def cublas(layers, only=None):
        for ents in layers:
            for name, NT, K, G, w, wp, x, y, rope in ents:
                if only is not None and name != only:
                    continue
                if G == 1:
                    torch.matmul(x, w.t(), out=y)
                else:
                    torch.bmm(x.view(B, G, K).transpose(0, 1), w.view(G, NT // G, K).transpose(1, 2))

    def per_layer_us(fn):
        side = torch.cuda.Stream()
        side.wait_stream(st)
        with torch.cuda.stream(side):
            fn()
        st.wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(st)
            graph.replay()
            e1.record(st)
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1) * 1e3 / copies)
        del graph
        return sorted(ts)[len(ts) // 2]

    merged = operands(PROJECTION_LAUNCHES)
    rows, tot_bytes = {}, 0
    for name, NT, K, G, _ in PROJECTION_LAUNCHES:
        nbytes = NT * K * 2 + B * G * K * 2 + B * NT * 2
        t = per_layer_us(lambda: native(merged, name))
        t_lib = per_layer_us(lambda: cublas(merged, name))
        rows[name] = {"us": round(t, 2), "gbs": round(nbytes / t / 1e3, 1), "cublas_us": round(t_lib, 2)}
        tot_bytes += nbytes
    tot = per_layer_us(lambda: native(merged))
    tot_lib_merged = per_layer_us(lambda: cublas(merged))
    del merged
    torch.cuda.empty_cache()
    separate = operands(PROJECTIONS)
    tot_lib = per_layer_us(lambda: cublas(separate))
    tot_sep = per_layer_us(lambda: native(separate))
    del separate
    torch.cuda.empty_cache()
    return {"batch": B, "us_per_layer": round(tot, 2), "cublas_us_per_layer": round(tot_lib, 2),
            "cublas_merged_us_per_layer": round(tot_lib_merged, 2), "native_separate_us_per_layer": round(tot_sep, 2),
            "bytes_per_layer": tot_bytes, "gbs": round(tot_bytes / tot / 1e3, 1),
            "frac": round(tot_bytes / tot / 1e3 / hbm, 4), "peak": hbm,
            "timing": f"graph of {copies} layers' projections with their own weights, back to back; "
                      f"median of {reps}; bytes = weights + activations in + result out; native = the four "
                      "launches DeviceAttention runs; cublas = the reference's nine matmuls",
            "kernels": rows}


def run_cfg1(args, rank, world, dev):
    """Config 1: the compressor emit path alone - batch 32, d 512, ratio 4,
    the [32, 4, 512] state (one slot per step, non-overlap form), softmax
    over slots, weighted sum, RMSNorm, emit every 4th step; 1000 steps from
    position 0, positions advanced on the device, one CUDA graph per step.
    Launch-bound by nature; reported as us per step."""
    import torch
    from dsv4attn import ops
    from dsv4attn.tables import PathArgs, rope_cos_sin
    B, d, r, steps = 32, 512, 4, 1000
    g = torch.Generator(device=dev).manual_seed(11 + rank)
    kv_row = torch.randn(B, d, device=dev, generator=g).to(torch.bfloat16)
    sc_row = torch.randn(B, d, device=dev, generator=g).to(torch.bfloat16)
    ape = 0.1 * torch.randn(r, d, device=dev, generator=g)
    gamma = 1 + 0.02 * torch.randn(d, device=dev, generator=g)
    kv_state = torch.zeros(B, r, d, device=dev)
    sc_state = torch.full((B, r, d), float("-inf"), device=dev)
    cos, sin = rope_cos_sin(PathArgs(), steps + 64, compressed=True, device=dev)
    cache = torch.zeros(B, steps // r + 2, d, dtype=torch.bfloat16, device=dev)
    pos = torch.zeros(B, dtype=torch.int32, device=dev)
    emitted = torch.zeros(B, dtype=torch.int32, device=dev)

    def one():
        ops.compressor_step(kv_row, sc_row, ape, kv_state, sc_state, gamma, cos, sin, cache, 0, pos, r, False,
                            emitted=emitted)
        ops.advance_positions(pos, None, r, 1)

    s_ = torch.cuda.Stream(dev)
    s_.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s_):
        one()
    torch.cuda.current_stream(dev).wait_stream(s_)
    torch.cuda.synchronize()
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        one()
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    best = None
    for _ in range(max(1, args.warmup) + 3):
        pos.zero_()
        kv_state.zero_()
        sc_state.fill_(float("-inf"))
        torch.cuda.synchronize()
        e0.record(st)
        for _ in range(steps):
            gr.replay()
        e1.record(st)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        best = ms if best is None else min(best, ms)
    us_step = best * 1e3 / steps
    n_emit = int((cache.float().abs().sum(-1) > 0).sum().item()) // B
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(B * 1e6 / us_step, 1), "unit": "tok/s", "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "ms_per_step": round(us_step / 1e3, 5),
            "us_per_step": round(us_step, 2), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded N(0,1) rows, ape N(0,0.1), gamma 1+N(0,0.02))",
            "config": {"workload": f"cfg1 compressor emit path: batch {B}, d {d}, ratio {r}, [32,4,512] state, "
                                   f"{steps} steps, emit every 4th ({n_emit} emitted rows per sequence)",
                       "global_batch": B, "parallelism": "replicas"},
            "note": "one compressor launch + one position advance per step, graph-replayed; launch-bound",
            **({"cpu_baseline": cpu_baseline_cfg1()} if world == 1 and not args.no_cpu else {})}),
            flush=True)


def run_cfg4(args, rank, world, dev):
    """Config 4: one prefill chunk of 4096 tokens x 64 heads x 512 against
    131072 prior tokens (32768 compressed entries): dense indexer, per-token
    top-2048, causal window 128, sink attention.  One step = one chunk of
    one layer; N GPUs each run their own chunk (queries shard with no
    exchange; "scaling": "weak").  Tensor-core bound: the roofline line is
    FLOP/s of the dominant kernel against the measured bf16 peak."""
    import torch
    import torch.distributed as dist
    from dsv4attn import ops
    from dsv4attn.prefill import PrefillChunk
    from dsv4attn.tables import PathArgs
    S, T, n_hist = 4096, 32768, 127
    base = 131072 - S
    pa = PathArgs(index_topk=args.topk)
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    n_raw = n_hist + S
    q = torch.randn(S, 64, 512, device=dev, generator=g).to(torch.bfloat16)
    kv = torch.randn(n_raw + T, 512, device=dev, generator=g).to(torch.bfloat16)
    iq = torch.randn(S, 64, 128, device=dev, generator=g).to(torch.bfloat16)
    ikeys = torch.randn(T, 128, device=dev, generator=g).to(torch.bfloat16)
    iw = 0.02 * torch.randn(S, 64, device=dev, generator=g)
    sink = torch.randn(64, device=dev, generator=g)
    out = torch.empty_like(q)
    ch = PrefillChunk(pa, S, T, dev)

    def chunk():
        ch.run(q, kv, n_raw, iq, ikeys, iw, sink, base, n_hist, T, out=out)

    def graph_of(fn):
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            fn()
        return gr

    g_all = graph_of(chunk)
    W = pa.window_size
    parts = {
        "indexer_score": lambda: ops.indexer_score(iq, ikeys, iw, T, out=ch.score, t_valid=ch.t_active),
        "indexer_topk": lambda: ops.indexer_topk(ch.score, ch.t_active, ch.k, n_raw, T=T, mask_mode=1,
                                                 out=ch.idx[:, W:], ws=ch.ws),
        "sparse_attn": lambda: ops.sparse_attn(q.view(1, S, 64, 512), kv.unsqueeze(0),
                                               ch.idx.view(1, S, W + ch.k), sink, pa.softmax_scale,
                                               out=out.view(1, S, 64, 512), ws=ch.ws, status=ch.status),
    }
    g_parts = {k: graph_of(f) for k, f in parts.items()}
    for _ in range(args.warmup):
        g_all.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(int(str(dev).split(":")[-1]))
    clocks.start()
    time.sleep(0.3)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0.record(st)
    for _ in range(args.steps):
        g_all.replay()
    e1.record(st)
    torch.cuda.synchronize()
    ms_total = e0.elapsed_time(e1)
    kt = {}
    for k, gr in g_parts.items():
        best = None
        for _ in range(3):
            e0.record(st)
            gr.replay()
            e1.record(st)
            e1.synchronize()
            v = e0.elapsed_time(e1)
            best = v if best is None else min(best, v)
        kt[k] = best
    clk = clocks.stop()
    if world > 1:
        t = torch.tensor([ms_total], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    ops.raise_for_status(ch.status, "cfg4 chunk")
    ms_chunk = ms_total / args.steps
    fl = ch.flops(T)
    pk = None
    pth = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(pth):
        with open(pth) as f:
            pk = json.load(f).get("bf16_tflops")
    peak = float(pk) if pk else 1590.0
    dom = "indexer_score" if kt["indexer_score"] >= kt["sparse_attn"] else "sparse_attn"
    dom_fl = fl["indexer"] if dom == "indexer_score" else fl["attention"]
    achieved = dom_fl / (kt[dom] * 1e-3) / 1e12
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(world * S / (ms_chunk / 1e3), 1), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_chunk, 4),
            "us_per_layer": round(ms_chunk * 1e3, 1), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1), indexer weights N(0,0.02))",
            "config": {"workload": f"cfg4 prefill chunk: {S} tokens x 64 heads x 512 over 131072 prior tokens "
                                   f"({T} compressed), per-token top-{ch.k} + causal window {W}, one layer",
                       "global_batch": world * S, "seq_len": 131072, "parallelism": f"query chunks x{world}",
                       "l2": "a chunk's working set (about 1 GB) exceeds L2"},
            "roofline": {"bound": "tensor", "kernel": dom, "achieved": round(achieved, 1), "peak": peak,
                         "unit": "TFLOP/s", "frac": round(achieved / peak, 4), "traffic": None,
                         "peak_kind": "measured (MEASURED_PEAKS.json bf16_tflops)" if pk else "fallback",
                         "flops": fl, "kernels_ms": {k: round(v, 3) for k, v in kt.items()}},
            "clocks": clk,
        }
        if world == 1 and not args.no_cpu:
            log("CPU baseline sample")
            line["cpu_baseline"] = cpu_baseline_cfg4()
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


class gpu_local_numa:
    """While active, the calling thread runs on the CPUs next to ``dev``
    (NVML's CPU affinity of the GPU, read-only use of NVML), so pinned host
    buffers allocated meanwhile get their pages on the GPU's own NUMA node
    (first touch); the previous affinity is restored on exit.  A no-op where
    NVML or sched_setaffinity is unavailable."""

    def __init__(self, dev):
        self.dev = dev
        self.prev = None
        self.cpus = None

    def __enter__(self):
        try:
            import torch
            import pynvml
            pr = torch.cuda.get_device_properties(self.dev)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            n = os.cpu_count() or 1
            words = pynvml.nvmlDeviceGetCpuAffinity(h, (n + 63) // 64)
            cpus = {64 * i + b for i, w in enumerate(words) for b in range(64) if (w >> b) & 1 and 64 * i + b < n}
            pynvml.nvmlShutdown()
            if cpus:
                self.prev = os.sched_getaffinity(0)
                os.sched_setaffinity(0, cpus)
                self.cpus = cpus
        except Exception:  # noqa: BLE001 - best effort: no NVML, no affinity API, no permission
            self.prev = None
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            os.sched_setaffinity(0, self.prev)
        return False


def measure_e2e(args, path, inputs, outs, dev, world):
    """Same metric through the public API with HOST buffers: every step copies
    all 43 layers' inputs from pinned host memory and reads all outputs back.
    Inputs and outputs of the whole step are packed (LayerInputs.packed, one
    flat output tensor) so each direction is one copy per step; the copies run
    on side streams, pipelined against the previous step's graph (two
    input/output buffer sets, one captured graph each)."""
    import torch
    from dsv4attn.layer import LayerInputs
    B, nl = args.batch, args.layers
    out_shape = (nl,) + tuple(outs[0].shape)
    # the pinned buffers live on this GPU's NUMA node (ranks spread over both
    # sockets' memory instead of all copying through one)
    with gpu_local_numa(dev) as numa:
        host_flat, host_in = LayerInputs.packed(path.args, B, nl, pin=True)
        host_out = torch.empty(out_shape, dtype=outs[0].dtype, pin_memory=True)
        host_flat.zero_()
        host_out.zero_()
    for h, x in zip(host_in, inputs):
        for a, b in zip(h.tensors(), x.tensors()):
            a.copy_(b)
    sets, graphs = [], []
    saved = path.graph
    for _ in range(2):
        dflat, dins = LayerInputs.packed(path.args, B, nl, device=dev)
        dflat.copy_(host_flat)
        dout = torch.empty(out_shape, dtype=outs[0].dtype, device=dev)
        sets.append((dflat, dout))
        path.graph = None
        graphs.append(path.capture(dins, list(dout.unbind(0)), warmup=0))
    path.graph = saved
    path.set_positions(args.ctx - 1)
    torch.cuda.synchronize()
    comp = torch.cuda.current_stream()
    h2d = torch.cuda.Stream(dev)
    d2h = torch.cuda.Stream(dev)
    in_ready = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    out_free = [torch.cuda.Event() for _ in range(2)]
    h2d_bytes = host_flat.numel()
    d2h_bytes = host_out.numel() * host_out.element_size()

    def issue(step):
        s = step & 1
        dflat, dout = sets[s]
        with torch.cuda.stream(h2d):
            if step >= 2:
                h2d.wait_event(done[s])          # graph of step-2 finished reading this set
            dflat.copy_(host_flat, non_blocking=True)
            in_ready[s].record(h2d)
        comp.wait_event(in_ready[s])
        if step >= 2:
            comp.wait_event(out_free[s])         # outputs of step-2 copied out
        graphs[s].replay()
        done[s].record(comp)
        with torch.cuda.stream(d2h):
            d2h.wait_event(done[s])
            host_out.copy_(dout, non_blocking=True)
            out_free[s].record(d2h)

    for i in range(3):
        issue(i)
    torch.cuda.synchronize()
    n = max(4, args.steps // 2)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    for i in range(n):
        issue(3 + i)
    comp.wait_stream(d2h)
    e1.record(comp)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    for g in graphs[1:]:
        del g
    return {"value": round(world * B * n / (ms / 1e3), 1), "unit": "tok/s", "h2d_bytes_per_step": h2d_bytes,
            "d2h_bytes_per_step": d2h_bytes, "steps": n, "ms_per_step": round(ms / n, 4),
            "host_numa": (f"pinned buffers allocated from the {len(numa.cpus)} CPUs local to the GPU"
                          if numa.cpus else "no NUMA placement (NVML affinity unavailable)"),
            "note": "pinned host inputs of all 43 layers H2D + all outputs D2H every step, pipelined with compute"}


if __name__ == "__main__":
    main()
