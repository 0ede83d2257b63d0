"""Decode-throughput benchmark of the B200 integer datapath (bit-exact int8).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c3] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N

Workload (config C3, the data-parallel config measured at 1/2/4/8 GPUs):
Qwen2.5-0.5B architecture with random N(0, 0.02) weights and QKV bias, quantized int8
per-channel; per GPU 128 independent sequences of 512 uniform-random prompt tokens, then
greedy decode with the reference runtime's launch rule (255 decode launches: the 256th
token is emitted without a launch because position 767 is the last of max_seq 768).
One *step* is that whole decode phase for the GPU's 128 sequences, starting from the
prefilled KV cache; prefill runs once, untimed.  Multi-GPU is data parallel: every rank
decodes its own 128 sequences with no collective ("weak" scaling); the timing is the max
over ranks.

Printed on rank 0: one JSON line with value (decode tokens/s over all GPUs, device-resident
tokens), e2e (the same metric through the C ABI host loop with host token buffers and a
host argmax read per launch), roofline of the dominant kernel, CPU baseline (the numpy
oracle port of the reference's golden model on this host), clocks and launch counts.

--impl reference times the reference algorithm's CPU implementation (the oracle port; the
reference's Python package does not exist on the GPU box) on a bounded sample of the same
workload, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="c3")
    ap.add_argument("--batch", type=int, default=None, help="sequences per GPU (default: the config's)")
    ap.add_argument("--prompt", type=int, default=None)
    ap.add_argument("--decode", type=int, default=None)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--artefacts", default=os.environ.get("LLX_ARTEFACTS", str(Path(tempfile.gettempdir()) / "llx_artefacts")))
    ap.add_argument("--e2e-steps", type=int, default=2)
    ap.add_argument("--cpu-decode", type=int, default=8, help="decode launches in the CPU baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--gemm-path", type=int, default=0)
    ap.add_argument("--lanes", type=int, default=1, help="concurrent decode lanes (sub-batches on own streams)")
    ap.add_argument("--tp", action="store_true",
                    help="tensor parallelism: all ranks form one group over the same sequences (C5 config)")
    return ap.parse_args()


# ---------------------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------------------
class _stdout_to_stderr:
    """Redirect file descriptor 1 to 2 (C libraries included) for the duration."""

    def __enter__(self):
        sys.stdout.flush()
        self.saved = os.dup(1)
        os.dup2(2, 1)

    def __exit__(self, *exc):
        sys.stdout.flush()
        os.dup2(self.saved, 1)
        os.close(self.saved)
class Dist:
    """One process per GPU (torchrun env): barrier and max-over-ranks timing.  backend
    "nccl" on GPUs; "gloo" serves the CPU tests of the same plumbing."""

    def __init__(self, want: int, backend: str = "nccl") -> None:
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.backend = backend
        self.pg = None
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist

            kw = {}
            if backend == "nccl":
                torch.cuda.set_device(self.local)
                kw["device_id"] = torch.device("cuda", self.local)
            # communicator set-up may print (e.g. NCCL's version line) on stdout, which must
            # carry only the result line: send fd 1 to stderr meanwhile
            with _stdout_to_stderr():
                dist.init_process_group(backend, timeout=datetime.timedelta(seconds=600), **kw)
                self.pg = dist
                self.barrier()
        if want != self.world and self.world > 1:
            raise SystemExit(f"--gpus {want} but WORLD_SIZE {self.world}")

    def barrier(self) -> None:
        if self.pg:
            self.pg.barrier()

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device="cuda" if self.backend == "nccl" else "cpu")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self) -> None:
        if self.pg:
            self.pg.destroy_process_group()
            self.pg = None


# ---------------------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int) -> None:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            ids = [v.strip() for v in vis.split(",") if v.strip()]
            self.device = ids[device] if device < len(ids) else device
        else:
            self.device = device
        self.proc = None
        self.lines: list[str] = []

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                smax = float(parts[1])
            except ValueError:
                continue
            for nm, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------------------
def workload(args):
    from llaccel_b200 import artefacts as A
    cfg = A.CONFIGS[args.config]
    w = dict(A.WORKLOADS[args.config])
    if args.batch:
        w["batch"] = args.batch
    if args.prompt:
        w["prompt"] = args.prompt
    if args.decode:
        w["decode"] = args.decode
    n_dec = min(w["decode"], max(0, cfg.max_seq - w["prompt"] - 1))
    return cfg, w, n_dec


def _wait_for(path: Path, what: str, limit_s: float = 1800.0) -> None:
    t0 = time.time()
    while not path.exists():
        if time.time() - t0 > limit_s:
            raise TimeoutError(f"{what} did not appear within {limit_s:.0f} s")
        time.sleep(0.5)


def make_artefact(args, dist: Dist) -> Path:
    """Rank 0 generates the config's artefact (once per artefacts dir); the other ranks wait
    for its manifest on the file system before the first collective."""
    from llaccel_b200 import artefacts as A
    root = Path(args.artefacts)
    root.mkdir(parents=True, exist_ok=True)
    d = root / f"{args.config}_s0_v2"
    if dist.rank == 0:
        A.ensure_artefact(args.config, root, seed=0, fusion=True, device="cuda")
    _wait_for(d / "manifest.json", "the artefact")
    dist.barrier()
    return d


def shard_artefact(full: Path, dist: Dist) -> Path:
    """This rank's graph of the tensor-parallel group over all ranks (written once)."""
    from llaccel_b200 import tp
    d = full.parent / f"{full.name}_tp{dist.world}" / f"r{dist.rank}"
    done = d / "done"
    if not done.exists():
        tp.shard(full, d, dist.rank, dist.world)
        done.write_text("ok")
    dist.barrier()
    return d


def tp_unique_id(dist: Dist) -> bytes:
    """NCCL unique id of the tensor-parallel group, made on rank 0 and broadcast."""
    from llaccel_b200.cuda_backend import tp_unique_id as make
    obj = [make() if dist.rank == 0 else None]
    if dist.pg:
        dist.pg.broadcast_object_list(obj, src=0)
    return obj[0]


def prompts_for(rank: int, B: int, L: int, vocab: int) -> np.ndarray:
    return np.random.default_rng(1000 + rank).integers(0, vocab, (B, L)).astype(np.int32)


def algorithmic_decode_bytes(m, prof: list[dict]) -> float:
    return float(sum(p["bytes"] for p in prof))


# configs whose full-prompt CPU prefill would take minutes: the CPU sample prefills a short
# prompt instead (decode cost per launch is dominated by the weights, not the context)
_SHORT_CPU_PROMPT = {"c4": 16, "c5": 16}


def cpu_baseline(qdir: Path, prompt: np.ndarray, n_dec: int, gpu_hist: np.ndarray | None, config: str = "",
                 gpu_short=None) -> dict:
    """Oracle port on this host: prefill one sequence (untimed), then time n_dec decode
    launches; compare the tokens with the GPU's decode history of the same sequence.  For
    the configs whose CPU sample prefills a short prompt, `gpu_short(prompt, n)` decodes
    the same short prompt on the GPU (n decode launches) for the comparison."""
    import os as _os
    from oracle import golden_oracle as O
    cores = _os.cpu_count() or 1
    o = O.OracleModel(qdir)
    if config in _SHORT_CPU_PROMPT:
        prompt = prompt[: _SHORT_CPU_PROMPT[config]]
        n_dec = min(n_dec, 4)
        gpu_hist = np.asarray(gpu_short([int(t) for t in prompt], n_dec)) if gpu_short else None
    toks = [int(t) for t in prompt]
    rows = o.prefill(toks)
    nxt = int(np.argmax(rows[-1][: o.vocab]))
    got = []
    t0 = time.perf_counter()
    pos = len(toks)
    for i in range(n_dec):
        lg = o.decode(nxt, pos + i)
        nxt = int(np.argmax(lg[: o.vocab]))
        got.append(nxt)
    dt = time.perf_counter() - t0
    parity = None
    if gpu_hist is not None:
        parity = bool(gpu_hist[: n_dec].tolist() == got)
    return {"value": n_dec / dt, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"1 sequence, {n_dec} decode launches at positions {pos}..{pos + n_dec - 1} after an untimed "
                      f"{len(toks)}-token prefill (numpy oracle of golden.py, BLAS threads = {cores}); "
                      f"the reference decodes batch sequences one after another, so this is its tokens/s",
            "parity_vs_gpu": parity}


def run_reference(args, dist: Dist) -> None:
    """--impl reference: the reference algorithm's CPU implementation, rank 0 only."""
    cfg, w, n_dec = workload(args)
    if dist.rank != 0:
        return
    from llaccel_b200 import artefacts as A
    root = Path(args.artefacts)
    qdir = A.ensure_artefact(args.config, root, seed=0, fusion=True, device="cuda" if _has_cuda() else "cpu")
    from oracle import golden_oracle as O
    cores = os.cpu_count() or 1
    o = O.OracleModel(qdir)
    prompt = prompts_for(0, 1, w["prompt"], cfg.vocab)[0].tolist()
    if args.config in _SHORT_CPU_PROMPT:
        prompt = prompt[: _SHORT_CPU_PROMPT[args.config]]
    rows = o.prefill(prompt)
    nxt = int(np.argmax(rows[-1][: o.vocab]))
    per_step = max(1, min(args.cpu_decode, n_dec))
    pos0 = len(prompt)

    def step():
        t = nxt
        for i in range(per_step):
            t = int(np.argmax(o.decode(t, pos0 + i)[: o.vocab]))

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    value = per_step * args.steps / dt
    sample = (f"1 of {w['batch']} sequences, {per_step} decode launches per step at positions "
              f"{pos0}..{pos0 + per_step - 1} after an untimed {len(prompt)}-token prefill; numpy oracle port of "
              f"golden.py (the reference package is not installed on the GPU box)")
    line = {"impl": "reference", "metric": f"decode tokens/s (bit-exact int8), {cfg.name}", "value": value,
            "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt / args.steps * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int8", "data": "synthetic",
            "config": {"workload": f"{cfg.name}: {w['batch']} seq/GPU, prompt {w['prompt']}, {n_dec} decode launches",
                       "parallelism": f"dp{args.gpus}"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _has_cuda() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def _by_kind(prof: list[dict]) -> dict:
    """Per-step kernel time summed by kind (linear steps split by output role)."""
    out: dict[str, list] = {}
    for p in prof:
        if p["ms"] <= 0:
            continue
        kind, _, name = p["label"].partition(":")
        if kind == "linear":
            role = name.split(".")[-1] if "." in name else name
            kind = f"linear.{role}"
        e = out.setdefault(kind, [0, 0.0, 0.0])
        e[0] += 1
        e[1] += p["ms"]
        e[2] += p["bytes"]
    return {k: {"n": v[0], "ms": round(v[1], 4), "GBs": round(v[2] / max(v[1], 1e-9) / 1e6, 1)}
            for k, v in sorted(out.items(), key=lambda kv: -kv[1][1])}


# plan step kind -> the kernel function that executes it on the decode path (M = 1 row per
# sequence, B >= 16 rows: tensor-core GEMMs)
_KERNEL_OF = {"linear": "k_linear_tc", "linear_group": "k_linear_tc", "gated": "k_linear_tc",
              "linear_partial": "k_linear_tc", "attention": "k_attention_decode", "rmsnorm": "k_rmsnorm",
              "rope_group": "k_rope_group", "rope": "k_rope", "add": "k_add", "mul": "k_mul", "silu": "k_silu",
              "quant": "k_quant", "kv_write": "k_kv_write", "embed": "k_embed", "argmax": "k_amax_finish",
              "requant": "k_requant", "allreduce": "ncclAllReduce"}


def _by_kernel(prof: list[dict], rows: int) -> dict:
    """Per-kernel-function totals of one decode launch of `rows` rows: launches, ms,
    algorithmic bytes.  Below 16 rows the linears run on the CUDA-core GEMV kernel."""
    out: dict[str, dict] = {}
    for p in prof:
        if p["ms"] <= 0:  # a step folded into its neighbour launches nothing
            continue
        kind = p["label"].partition(":")[0]
        k = _KERNEL_OF.get(kind, kind)
        if k == "k_linear_tc" and rows < 16:
            k = "k_gemv"
        e = out.setdefault(k, {"n": 0, "ms": 0.0, "bytes": 0.0})
        e["n"] += 1
        e["ms"] += p["ms"]
        e["bytes"] += p["bytes"]
    return out


def _committed_traffic(config: str, batch: int, kernel: str):
    """DRAM traffic per launch of `kernel` from a committed ncu summary, if one exists for
    this config and batch (profiles/traffic.json, written from an ncu capture)."""
    f = REPO / "profiles" / "traffic.json"
    if not f.exists():
        return None
    for e in json.loads(f.read_text()).get("entries", []):
        if e.get("config") == config and e.get("batch") == batch and e.get("kernel") == kernel:
            return e
    return None


_ARCH = {"c1": "tiny Llama", "c2": "SmolLM2-135M arch", "c3": "Qwen2.5-0.5B arch, QKV bias",
         "c4": "Qwen3-0.6B arch, q/k norm", "c5": "Llama-3-8B arch"}


def run_ours(args, dist: Dist) -> None:
    import torch
    from llaccel_b200 import build
    build.build()
    from llaccel_b200.cuda_backend import CudaLanes

    cfg, w, n_dec = workload(args)
    dev = dist.local
    torch.cuda.set_device(dev)
    qdir = make_artefact(args, dist)
    B, L = w["batch"], w["prompt"]
    lanes = args.lanes if B % args.lanes == 0 else 1
    model_kw = {}
    if args.tp:
        # one tensor-parallel group: every rank holds all B sequences and 1/world of each layer
        full = qdir
        qdir = shard_artefact(full, dist)
        model_kw["tp"] = (dist.rank, dist.world, tp_unique_id(dist))
        lanes = 1
        prompts = prompts_for(0, B, L, cfg.vocab)
    else:
        full = qdir
        prompts = prompts_for(dist.rank, B, L, cfg.vocab)
    seq_groups = 1 if args.tp else dist.world  # independent sequence sets decoded per step
    # prefill launches of up to 512 rows per sequence, fewer when B*rows would exceed 64K rows
    max_rows = max(16, min(L, 512, (65536 // B) // 16 * 16))
    with _stdout_to_stderr():  # a tensor-parallel model opens its NCCL communicator here
        m = CudaLanes(qdir, batch=B, lanes=lanes, device=dev, max_rows=max_rows, gemm_path=args.gemm_path,
                      **model_kw)
    t0 = time.perf_counter()
    recs = m.generate_batch(prompts.tolist(), 0, with_logits=False)  # prefill (untimed)
    prefill_s = time.perf_counter() - t0
    first = np.array([r["argmax_per_step"][-1] for r in recs], np.int32)
    streams = [torch.cuda.ExternalStream(h, device=dev) for h in m.streams()]

    def step():
        m.set_tokens(first)
        m.decode_async(L, n_dec)

    for _ in range(args.warmup):
        step()
    m.sync()
    hist = m.history(n_dec)
    clocks = ClockSampler(dev)
    dist.barrier()
    torch.cuda.synchronize(dev)
    clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ends = [torch.cuda.Event() for _ in streams]
    # every lane stream starts after e0; e1 follows the last lane; set_tokens synchronises
    # only its own lane's stream, so the lanes' decode chains overlap on the GPU
    e0.record(streams[0])
    for sl in streams[1:]:
        sl.wait_event(e0)
    for _ in range(args.steps):
        step()
    for ev, sl in zip(ends, streams):
        ev.record(sl)
        streams[0].wait_event(ev)
    e1.record(streams[0])
    m.sync()
    torch.cuda.synchronize(dev)
    dist.barrier()
    clock = clocks.stop()
    ms = e0.elapsed_time(e1)
    ms_max = dist.max(ms)
    total_tokens = seq_groups * B * n_dec * args.steps
    value = total_tokens / (ms_max / 1e3)
    # the decode history must be identical every step (same prompt state, same tokens)
    hist2 = m.history(n_dec)
    deterministic = bool(np.array_equal(hist, hist2))

    # e2e: the C-ABI host loop per lane (one host thread each), host token buffers in, host
    # argmax out, per decode launch
    import threading as th
    from llaccel_b200.cuda_backend import _check, _p32
    e2e_steps = max(1, args.e2e_steps)
    per = B // lanes
    outs = [None] * lanes

    trace = [None] * lanes

    def run_lane(li):
        mm = m.models[li]
        lib, sess = mm.lib, mm._sess
        am = np.zeros(per, np.int32)
        cur = None
        tr = np.zeros((n_dec, per), np.int32)
        for _ in range(e2e_steps):
            cur = first[li * per : (li + 1) * per].reshape(per, 1).copy()  # never a view of `first`
            for i in range(n_dec):
                _check(lib, lib.llx_run(sess, _p32(cur), 1, L + i, None, 0, None, _p32(am)))
                cur[:, 0] = am
                tr[i] = am
        outs[li] = cur[:, 0].copy()
        trace[li] = tr

    dist.barrier()
    t0 = time.perf_counter()
    threads = [th.Thread(target=run_lane, args=(li,)) for li in range(lanes)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    e2e_s = dist.max(time.perf_counter() - t0)
    e2e_trace = np.concatenate(trace, axis=1)
    e2e_ok = bool(np.array_equal(e2e_trace, hist))
    bad_steps = np.nonzero((e2e_trace != hist).any(axis=1))[0]
    e2e_diag = {"mismatch_steps": int(len(bad_steps)), "first_bad_step": int(bad_steps[0]) if len(bad_steps) else None,
                "mismatch_tokens": int((e2e_trace != hist).sum())}
    if len(bad_steps):
        e2e_diag["step0_e2e"] = e2e_trace[0, :8].tolist()
        e2e_diag["step0_dev"] = hist[0, :8].tolist()
    e2e_value = seq_groups * B * n_dec * e2e_steps / e2e_s
    h2d = n_dec * (B * 4 + 8 * lanes)
    d2h = n_dec * (B * 4 + 8 * lanes)

    # per-kernel profile of one lane at the middle decode position (roofline of the dominant kernel)
    m0 = m.models[0]
    pos_mid = L + n_dec // 2
    prof = m0.profile_decode(pos_mid, iters=20)
    launches_per_step = m0.decode_launches_per_step()
    step_ms_sum = sum(p["ms"] for p in prof)
    kern = _by_kernel(prof, B // lanes)
    dom_name = max(kern, key=lambda k: kern[k]["ms"])
    dom = kern[dom_name]
    peaks = {}
    pk = REPO / "MEASURED_PEAKS.json"
    if pk.exists():
        peaks = json.loads(pk.read_text())
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    # whole decode launch (all lanes): algorithmic bytes = weights once per lane + KV + acts
    step_bytes = sum(p["bytes"] for p in prof) * lanes
    step_ms_graph = ms_max / args.steps / n_dec
    whole = {"decode_launch_ms": step_ms_graph, "algorithmic_bytes_per_launch": step_bytes,
             "achieved_gbs": step_bytes / (step_ms_graph / 1e3) / 1e9,
             "frac_of_hbm": step_bytes / (step_ms_graph / 1e3) / 1e9 / hbm, "lane_kernels_sum_ms": step_ms_sum,
             "lanes": lanes}
    # Per-kernel time inside the decode graph: each step is timed alone (CUDA events around one
    # launch after an L2 flush: its inputs come from HBM, as in the chain) for its SHARE of the
    # launch; the share times the graph replay's measured launch time is the kernel's time in
    # the graph.  The isolated time also carries the single launch's start-up latency, which
    # the graph hides behind the previous kernel (programmatic dependent launch), so it is
    # reported beside (us_isolated), not used for the roofline.  The dominant kernel = the
    # function with the largest share; achieved = its algorithmic bytes per launch / its time.
    graph_ms = step_ms_graph  # one lane's kernels span the launch (lanes run concurrently)
    for v in kern.values():
        v["ms_graph"] = v["ms"] / step_ms_sum * graph_ms
    dom_gbs = dom["bytes"] / (dom["ms_graph"] / 1e3) / 1e9
    traffic = _committed_traffic(cfg.name, B, dom_name)
    roof = {"bound": "hbm", "kernel": dom_name, "achieved": dom_gbs, "peak": hbm, "unit": "GB/s",
            "frac": dom_gbs / hbm, "peak_source": peak_src,
            "time_source": "share of the decode launch (each kernel timed alone after an L2 flush) x the graph "
                           "replay's launch time",
            "traffic": traffic["bytes_per_launch"] if traffic else None,
            "traffic_source": traffic["source"] if traffic else None,
            "launches_per_decode_launch": dom["n"], "bytes_per_launch": dom["bytes"] / dom["n"],
            "ms_per_launch": dom["ms_graph"] / dom["n"], "ms_per_launch_isolated": dom["ms"] / dom["n"],
            "share_of_step": dom["ms"] / step_ms_sum,
            "by_kernel": {k: {"n": v["n"], "share": round(v["ms"] / step_ms_sum, 4),
                              "us_per_launch": round(1e3 * v["ms_graph"] / v["n"], 2),
                              "us_isolated": round(1e3 * v["ms"] / v["n"], 2),
                              "GBs": round(v["bytes"] / (v["ms_graph"] / 1e3) / 1e9, 1),
                              "frac": round(v["bytes"] / (v["ms_graph"] / 1e3) / 1e9 / hbm, 4)}
                          for k, v in sorted(kern.items(), key=lambda kv: -kv[1]["ms"])}}

    base = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        from llaccel_b200.cuda_backend import CudaModel

        def gpu_short(prompt, n):
            # one sequence on the loaded weights (own session): n decode launches after the prompt
            with CudaModel(qdir, batch=1, device=dev, max_rows=64, share=m.models[0]) as one:
                return one.generate(prompt, n + 1)["generated"][1:]

        base = cpu_baseline(full, prompts[0], min(args.cpu_decode, n_dec), hist[:, 0], cfg.name, gpu_short)
    line = {
        "metric": f"decode tokens/s (bit-exact int8), {cfg.name}",
        "value": value, "unit": "tokens/s", "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_max / args.steps, "higher_is_better": True,
        "scaling": "strong" if args.tp else "weak", "vs_baseline": None,
        "dtype": "int8", "data": "synthetic",
        "config": {"workload": f"{cfg.name} ({_ARCH.get(cfg.name, cfg.name)}) decode: {B} seq"
                               f"{'' if args.tp else '/GPU'}, prompt {L}, {n_dec} decode launches/step",
                   "global_batch": B * seq_groups, "seq_len": L + n_dec, "prompt": L, "decode_launches": n_dec,
                   "parallelism": f"tp{dist.world}" if args.tp else f"dp{dist.world}", "lanes_per_gpu": lanes,
                   "l2": f"inputs larger than L2: every decode launch streams "
                         f"{step_bytes / 1e9:.2f} GB of weights + KV per GPU",
                   "prefill_s_untimed": prefill_s},
        "roofline": roof, "decode_launch": whole,
        "cpu_baseline": base,
        "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "steps": e2e_steps, "path": f"llx_run per decode launch (C ABI, host buffers), {lanes} host threads",
                "tokens_match_device_loop": e2e_ok, **e2e_diag},
        "clocks": clock,
        "gpu_launches": launches_per_step * lanes * n_dec * args.steps,
        "determinism": deterministic,
        "profile_by_kind": _by_kind(prof),
        "profile_top": [{"k": p["label"], "ms": round(p["ms"], 5), "GBs": round(p["bytes"] / max(p["ms"], 1e-9) / 1e6, 1)}
                        for p in sorted(prof, key=lambda p: -p["ms"])[:6]],
    }
    if dist.rank == 0:
        print(json.dumps(line), flush=True)
    m.close()


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        # the reference arm is CPU work on rank 0; other ranks exit without work
        rank = int(os.environ.get("RANK", "0"))
        if rank == 0:
            run_reference(args, Dist(1) if int(os.environ.get("WORLD_SIZE", "1")) == 1 else _NoDist())
        return
    if args.tp:
        # The tensor-parallel all-reduces are 4 MB int32 buffers per op: latency-bound, and
        # NCCL's low-latency protocol measured faster on them (C5 TP2 24.9K -> 26.6K tok/s).
        # NCCL reads it once, at the process's first communicator, so it is set here.
        os.environ.setdefault("NCCL_PROTO", "LL")
    dist = Dist(args.gpus)
    try:
        run_ours(args, dist)
    finally:
        dist.close()


class _NoDist:
    rank, world, local = 0, 1, 0

    def barrier(self):
        pass


if __name__ == "__main__":
    main()
