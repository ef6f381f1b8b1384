"""EM-iteration throughput benchmark (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

A step is one full soft-EM iteration (prepare, fused E+M statistics, one
allreduce when N > 1, finalize) over the configuration's whole synthetic
dataset, which is resident in HBM and sharded by rows across the ranks
(strong scaling: the total N is the configuration's N at every GPU count).
Default workload: configs[4] of BASELINE.json, the largest configuration that
fits one B200 and the one the north star's 1 -> 8 GPU scaling target names --
spherical GMM, bf16 X with fp32 accumulation, N = 200,000,000, D = 128,
K = 8192 (51.2 GB of X).  ``--config 1`` .. ``--config 3`` run the others.

``value``  samples/s per EM iteration, device-timed (CUDA events on the compute
           stream, barrier + synchronize on both sides, max over ranks).
``e2e``    the same metric through the public streamed API
           (``large_n.em_fit_streamed``, one call of K iterations): X in
           pinned host memory, every iteration copies its rows host->device
           (double-buffered copy stream overlapping the kernels) and reads the
           iteration's lower bound back to the host.
``roofline`` the dominant kernel launch (gmmxx_em_accumulate) against the
           measured bf16 tensor peak, algorithmic FLOPs only; ``kernel`` names
           the statistics kernels the library reports it launched.
``cpu_baseline`` the reference's own torch CPU implementation
           (``gmmxx.torch_fallback.batch_gmm_*_torch_native``, the unmodified
           package installed under baseline/_ref) on the host cores, on a
           bounded row sample, rank 0 at N = 1.

``--impl reference`` times that reference CPU path alone, per step on a
bounded row sample.  Only when baseline/_ref cannot be imported does either
leg fall back to the numpy restatement under oracle/ (``kind: "port"``).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)


def algorithmic_flops(cov: str, n: int, d: int, k: int) -> float:
    """Per-iteration algorithmic FLOPs of the E-step logit contraction plus the
    M-step statistics contraction (expanded-distance form, one pass each)."""
    if cov == "diag":
        return 2.0 * n * k * (2 * d) + 2.0 * n * k * (2 * d + 1)
    if cov == "spherical":
        return 2.0 * n * k * d + 2.0 * n * k * (d + 2)
    if cov == "tied":
        return 2.0 * n * k * d + 2.0 * n * d * d + 2.0 * n * k * (d + 1)
    q = d * (d + 1) // 2
    return 2.0 * n * k * (d + q) + 2.0 * n * k * (1 + d + q)


def launches_per_iteration(cfg, tc_path: bool, approx: bool = False) -> int:
    """Kernels of this library launched per EM iteration: prep_weights +
    prep_table (+ 2 Cholesky kernels for tied / full), the statistics kernels,
    finalize (per component, then per problem).  Statistics: 3 (pack,
    tensor-core kernel, reduce; or rows, mstep, reduce; or the two approximate
    top-k passes and reduce); 2 for the one-pass K <= 64 kernel and its
    reduce; for spherical K > 1024 the grouped passes: pack, G1 row-partial
    launches, combine, log-likelihood sum, G2 x (M-step launch + reduce) --
    G1 = G2 = the groups of 4 chunks on em_tc_kernel (D = 64, or the legacy
    layout); on the diag-kernel layout (D = 128) G1 counts groups of 2
    chunks (the row-statistics pass) and G2 groups of 4."""
    prep = 2 + (2 if cfg.cov_type in ("tied", "full") else 0)
    stats = 2 if (not tc_path and not approx and cfg.K <= 64) else 3  # K <= 64: one-pass kernel + reduce
    if tc_path and cfg.cov_type == "spherical" and cfg.K > 1024:
        nch = (cfg.K + 127) // 128
        g2 = (nch + 3) // 4  # groups of 4 chunks (512 components)
        new_layout = cfg.D == 128 and os.environ.get("GMMXX_B200_SPH_KERNEL") != "legacy"
        g1 = (nch + 1) // 2 if new_layout else g2
        stats = 3 + g1 + 2 * g2
    return prep + stats + 2


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        return {"hbm_gbs": p["hbm_gbs"], "bf16": p["bf16_tflops"], "bf16_sus": p["bf16_tflops_sustained"],
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sus": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


REF_PATH = os.path.join(ROOT, "baseline", "_ref")
# rows per problem of one timed reference sample (about 1-3 s of host work on 16 threads)
REF_ROWS = {0: 100_000, 1: 200_000, 2: 500_000, 3: 16_384, 4: 20_000}
# rows per problem of the cpu_baseline leg (about 10-30 s)
CPU_ROWS = {0: 100_000, 1: 1_000_000, 2: 2_000_000, 3: 65_536, 4: 100_000}


def reference_module():
    """The reference's own torch implementation (gmmxx.torch_fallback of the
    unmodified package installed under baseline/_ref), or (None, reason)."""
    if not os.path.isdir(os.path.join(REF_PATH, "gmmxx")):
        return None, "baseline/_ref not installed"
    if REF_PATH not in sys.path:
        sys.path.insert(0, REF_PATH)
    try:
        from gmmxx import torch_fallback
    except Exception as exc:  # report, never fake
        return None, repr(exc)
    return torch_fallback, None


def cpu_sample(cfg, mix, init, rows: int, iters: int = 1, approx_top_k=None):
    """One timed fit of ``iters`` EM iterations on ``rows`` rows per problem,
    on the host cores, by the reference's own torch CPU path
    (batch_gmm_*_torch_native from baseline/_ref, tol=0, no Triton, same
    initial parameters as the GPU arm, labels off); the numpy port of it under
    oracle/ only when the reference cannot be imported."""
    import torch

    from gmmxx_b200 import synthetic

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    x = synthetic.sample_rows(cfg, mix, rows, torch.device("cpu"), seed=12345).float()
    means, cov, w = init
    tf, why = reference_module()
    sample = f"{cfg.B}x{rows} rows of config {cfg.index}, {iters} EM iteration(s), float32"
    if tf is not None:
        fn = {"spherical": tf.batch_gmm_Spherical_torch_native, "diag": tf.batch_gmm_Diagonal_torch_native,
              "tied": tf.batch_gmm_Tied_torch_native, "full": tf.batch_gmm_Full_torch_native}[cfg.cov_type]
        kw = dict(max_iters=iters, tol=0.0, init_means=torch.from_numpy(means), init_variances=torch.from_numpy(cov),
                  init_weights=torch.from_numpy(w), reg_covar=1e-6, compute_labels=False, approx_top_k=approx_top_k)
        if cfg.cov_type == "spherical":
            kw.update(gmm_use_triton_estep=False, gmm_use_triton_streaming_update=False)
        else:
            kw.update(gmm_use_triton=False)
        t0 = time.perf_counter()
        fn(x, cfg.K, **kw)
        dt = time.perf_counter() - t0
        return {"value": rows * cfg.B * iters / dt, "unit": "samples/s", "cores": threads, "kind": "reference",
                "sample": f"{sample}, the reference's {fn.__name__} (torch {torch.__version__} CPU, "
                          f"{threads} threads), {dt:.2f} s"}
    import oracle

    t0 = time.perf_counter()
    oracle.fit(cfg.cov_type, x.numpy(), cfg.K, iters, 0.0, means, cov, w, compute_labels=False,
               approx_top_k=approx_top_k)
    dt = time.perf_counter() - t0
    return {"value": rows * cfg.B * iters / dt, "unit": "samples/s", "cores": threads, "kind": "port",
            "sample": f"{sample}, numpy port under oracle/ ({dt:.2f} s); reference not importable: {why}"}


def run_reference(args, cfg):
    """--impl reference: the reference's torch CPU path timed per step on a
    bounded row sample (rank 0 only; other ranks exit without work)."""
    from gmmxx_b200 import synthetic

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    mix = synthetic.mixture_params(cfg)
    init = synthetic.initial_params(cfg, mix)
    rows = args.ref_rows or REF_ROWS[cfg.index]
    for _ in range(args.warmup):
        cpu_sample(cfg, mix, init, rows, approx_top_k=args.approx_top_k)
    runs = [cpu_sample(cfg, mix, init, rows, approx_top_k=args.approx_top_k) for _ in range(args.steps)]
    v = statistics.median(r["value"] for r in runs)
    line = {
        "impl": "reference", "metric": "EM samples/s per iteration", "value": v, "unit": "samples/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * rows * cfg.B / v,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": workload_config(cfg, args),
        "cpu_baseline": {"value": v, "unit": "samples/s", "cores": runs[0]["cores"], "kind": runs[0]["kind"],
                         "sample": f"per step: {runs[0]['sample']}"},
        "e2e": {"value": v, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_infer(args, cfg, x, means, cov, weights):
    """--infer: one inference call per step on the rows already in HBM, timed
    with CUDA events on the launching stream (the output buffer of
    predict_proba is allocated once).  Roofline: algorithmic logit FLOPs
    against the bf16 peak for labels / score_samples, and the output bytes
    against HBM for predict_proba (its output of K floats per row bounds it)."""
    import torch

    from gmmxx_b200 import engine

    from gmmxx_b200 import _native as nat

    B, N, D, K = cfg.B, x.shape[-2], cfg.D, cfg.K
    dev = x.device
    tc_path = nat.accumulate_path(engine.cov_code(cfg.cov_type), nat.BFLOAT16 if x.dtype == torch.bfloat16
                                  else nat.FLOAT32, B, N, D, K) == 1
    nch = (K + 127) // 128  # spherical D = 128: the diag kernel's layout for K <= 512 and K > 1024
    sph_new = (cfg.cov_type == "spherical" and D == 128 and (nch <= 4 or nch > 8)
               and os.environ.get("GMMXX_B200_SPH_KERNEL") != "legacy")
    out = torch.empty((B, N, K), dtype=torch.float32, device=dev) if args.infer == "proba" else None
    call = {"predict": lambda: engine.assign(cfg.cov_type, x, means, cov, weights),
            "score": lambda: engine.score_samples(cfg.cov_type, x, means, cov, weights),
            "proba": lambda: engine.predict_proba(cfg.cov_type, x, means, cov, weights, out=out)}[args.infer]
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for e0, e1 in evs:
        e0.record(stream)
        call()
        e1.record(stream)
    torch.cuda.synchronize()
    ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs)
    rows = B * N
    fe = {"spherical": D, "diag": 2 * D, "tied": D, "full": D + D * (D + 1) // 2}[cfg.cov_type]
    flops = rows * 2.0 * K * fe  # the logits once (the algorithmic minimum, whatever the passes)
    out_bytes = rows * {"predict": 8, "score": 4, "proba": 4 * K}[args.infer]
    in_bytes = rows * D * x.element_size()
    peaks = load_peaks()
    tflops = flops / (ms / 1e3) / 1e12
    gbs = (out_bytes + in_bytes) / (ms / 1e3) / 1e9
    hbm = args.infer == "proba"
    line = {
        "metric": {"predict": "labels rows/s", "score": "score_samples rows/s", "proba": "predict_proba rows/s"}[
            args.infer],
        "value": rows / (ms / 1e3), "unit": "rows/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "dtype": "f32", "data": "synthetic",
        "config": workload_config(cfg, args),
        "kernel": ("em_tc_diag_kernel, inference mode (tensor cores)" if (cfg.cov_type == "diag" or sph_new) and tc_path
                   else "em_tc_kernel, per-row inference passes (tensor cores)" if tc_path
                   else "rows_kernel (CUDA cores)"),
        "roofline": {"bound": "hbm" if hbm else "tensor", "achieved": gbs if hbm else tflops,
                     "peak": peaks["hbm_gbs"] if hbm else peaks["bf16"], "unit": "GB/s" if hbm else "TFLOP/s",
                     "frac": (gbs / peaks["hbm_gbs"]) if hbm else (tflops / peaks["bf16"]),
                     "peak_source": peaks["source"],
                     "algorithmic_flops": flops, "bytes": out_bytes + in_bytes, "achieved_tflops": tflops},
    }
    print(json.dumps(line), flush=True)


def workload_config(cfg, args):
    names = {0: "configs[0] spherical", 1: "configs[1] diag", 2: "configs[2] tied", 3: "configs[3] full",
             4: "configs[4] spherical large-K"}
    conf = {"workload": f"{names[cfg.index]} GMM EM iteration", "covariance_type": cfg.cov_type,
            "x_dtype": str(cfg.dtype).replace("torch.", ""), "B": cfg.B, "N": cfg.N, "D": cfg.D, "K": cfg.K,
            "parallelism": f"dp{args.gpus} (rows sharded, stats allreduce)",
            "l2": "inputs larger than L2 (126 MB); no flush needed"}
    if args.approx_top_k:
        conf["workload"] = f"{names[cfg.index]} GMM approximate top-{args.approx_top_k} EM iteration"
        conf["approx_top_k"] = args.approx_top_k
    return conf


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", type=int, default=4)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--n", type=int, default=0, help="override total N (smaller runs)")
    ap.add_argument("--ref-rows", type=int, default=0,
                    help="rows per problem of each --impl reference step (default: per configuration)")
    ap.add_argument("--cpu-rows", type=int, default=0,
                    help="rows per problem of the cpu_baseline sample (default: per configuration, 10-30 s)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--chunk-rows", type=int, default=1 << 22, help="rows per host->device chunk of the e2e leg")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--infer", choices=["predict", "score", "proba"], default=None,
                    help="time an inference call (labels / score_samples / predict_proba) instead of EM")
    ap.add_argument("--approx-top-k", type=int, default=None,
                    help="time approximate top-k EM (CUDA-core kernels) instead of exact EM; no e2e leg")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.approx_top_k:
        args.no_e2e = True

    from gmmxx_b200 import synthetic

    cfg = synthetic.CONFIGS[args.config]
    if args.n:
        cfg = synthetic.Config(cfg.index, cfg.cov_type, cfg.dtype, cfg.B, args.n, cfg.D, cfg.K, cfg.iters)
    if args.impl == "reference":
        run_reference(args, cfg)
        return

    import torch
    import torch.distributed as dist

    from gmmxx_b200 import _native as nat
    from gmmxx_b200 import engine, large_n

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
        comm = engine.Comm()
    nat.load()

    mix = synthetic.mixture_params(cfg)
    init_means, init_cov, init_w = synthetic.initial_params(cfg, mix)
    n_local = cfg.N // world + (1 if rank < cfg.N % world else 0)
    x = synthetic.sample_rows(cfg, mix, n_local, dev, seed=1000 + rank)
    torch.cuda.synchronize()

    means, cov, weights, _ = engine.initial_parameters(
        cfg.cov_type, x, cfg.K, torch.from_numpy(init_means), torch.from_numpy(init_cov),
        torch.from_numpy(init_w), 1e-6)
    if args.infer:
        if world > 1:
            raise SystemExit("--infer runs on one GPU")
        run_infer(args, cfg, x, means, cov, weights)
        return
    top_k = engine.resolve_approx_top_k(args.approx_top_k, cfg.K)
    ops = engine.CudaOps(cfg.cov_type, x, cfg.K, top_k)
    B, D, K = cfg.B, cfg.D, cfg.K
    nstat = B * K * ops.stat_width
    # the statistics and (last slot, multi-rank only) the log-likelihood: one collective per step
    pack = torch.zeros((nstat + (1 if comm else 0),), dtype=torch.float32, device=dev)
    stats = pack[:nstat].view(B, K, ops.stat_width)
    ll = torch.zeros((1,), dtype=torch.float64, device=dev)
    lb = torch.zeros((1,), dtype=torch.float32, device=dev)
    xx = None
    if cfg.cov_type == "tied":
        xx = torch.zeros((B, D, D), dtype=torch.float32, device=dev)
        ops.xx_total(xx)
        if comm:
            comm.allreduce_(xx)
    stream = torch.cuda.current_stream(dev)
    ev_acc = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]

    def step(i=None):
        ops.prepare(means, cov, weights, 1e-6, 1e-8)
        stats.zero_()
        ll.zero_()
        if i is not None:
            ev_acc[i][0].record(stream)
        ops.accumulate(stats, ll)
        if i is not None:
            ev_acc[i][1].record(stream)
        if comm:
            pack[nstat:].copy_(ll)
            comm.allreduce_(pack)
            ll.copy_(pack[nstat:])
        ops.finalize(cfg.N, stats, ll, xx, 1e-6, 1e-8, means, cov, weights, lb)

    for _ in range(args.warmup):
        step()
    sampler = ClockSampler(local)
    if comm:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record(stream)
    for i in range(args.steps):
        step(i)
    t_end.record(stream)
    torch.cuda.synchronize()
    if comm:
        dist.barrier()
    clocks = sampler.stop()
    ms = t_start.elapsed_time(t_end) / args.steps
    acc_ms = sum(a.elapsed_time(b) for a, b in ev_acc) / args.steps
    ms_t = torch.tensor([ms, acc_ms], dtype=torch.float64, device=dev)
    if comm:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms, acc_ms = float(ms_t[0]), float(ms_t[1])
    ops.check_status()
    kernel_path = ops.kernel_path()
    tc_path = top_k is None and ops.paths == {1}
    value = cfg.N * cfg.B / (ms / 1e3)

    # --- end to end through the public streamed API (host-resident X) -------
    e2e = None
    if not args.no_e2e and cfg.B == 1:
        x_host = torch.empty((1, n_local, D), dtype=cfg.dtype, pin_memory=True)
        x_host.copy_(x)
        del x, ops
        torch.cuda.empty_cache()
        streamer = large_n.ChunkStreamer(x_host, args.chunk_rows, dev)
        init_t = [torch.from_numpy(a) for a in (init_means, init_cov, init_w)]

        def e2e_fit(iters):
            # tol > 0 makes the loop read each iteration's lower bound back to the
            # host (the step's result); 1e-30 never stops these fits early
            return large_n.em_fit_streamed(cfg.cov_type, x_host, K, device=dev, chunk_rows=args.chunk_rows,
                                           max_iters=iters, tol=1e-30, init_means=init_t[0],
                                           init_variances=init_t[1], init_weights=init_t[2], reg_covar=1e-6,
                                           compute_labels=False, streamer=streamer, comm=comm)

        e2e_fit(args.warmup)
        if comm:
            dist.barrier()
        torch.cuda.synchronize()
        streamer.h2d_bytes = 0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        _, m2, c2, w2, info2 = e2e_fit(args.steps)
        host_out = [t.cpu() for t in (m2, c2, w2)]
        e1.record(stream)
        torch.cuda.synchronize()
        if comm:
            dist.barrier()
        it2 = info2["n_iter"]
        ems = torch.tensor([e0.elapsed_time(e1) / it2], dtype=torch.float64, device=dev)
        if comm:
            dist.all_reduce(ems, op=dist.ReduceOp.MAX)
        e2e = {"value": cfg.N * cfg.B / (float(ems[0]) / 1e3), "unit": "samples/s",
               "h2d_bytes_per_step": streamer.h2d_bytes // it2,
               "d2h_bytes_per_step": 4 + sum(h.numel() * h.element_size() for h in host_out) // it2,
               "iterations": it2, "kernel_path": info2["kernel_path"],
               "path": f"gmmxx_b200.large_n.em_fit_streamed, one call of {it2} iterations over pinned host X "
                       f"({args.chunk_rows}-row double-buffered chunks), lower bound read back every iteration"}

    if rank == 0:
        peaks = load_peaks()
        flops = algorithmic_flops(cfg.cov_type, n_local * cfg.B, D, K)
        achieved = flops / (acc_ms / 1e3) / 1e12
        long_run = ms * args.steps > 1000.0
        peak = peaks["bf16_sus"] if long_run else peaks["bf16"]
        traffic = None
        tpath = os.path.join(ROOT, "profiles", "traffic.json")
        if os.path.exists(tpath) and top_k is None:  # the captured traffic is the exact-EM kernel's
            with open(tpath) as f:
                tr = json.load(f).get(f"config{cfg.index}")
            if tr and tr.get("path", "tensor-core") == kernel_path:
                traffic = (tr["read_bytes_per_row"] + tr.get("write_bytes_per_row", 0.0)) * n_local * cfg.B + \
                    tr["write_bytes_per_launch"]
        nch = (K + 127) // 128
        sph_new = D == 128 and (nch <= 4 or nch > 8) and os.environ.get("GMMXX_B200_SPH_KERNEL") != "legacy"
        kernel_names = {"diag": "em_tc_diag_kernel", "tied": "em_tc_diag_kernel<tied>",
                        "spherical": (("em_tc_diag_kernel<spherical> row statistics + em_tc_sph_ext_kernel"
                                       if os.environ.get("GMMXX_B200_SPH_PASS2") != "diag" else
                                       "em_tc_diag_kernel<spherical> (row-statistics + external-lse passes)")
                                      if sph_new and nch > 8 else "em_tc_diag_kernel<spherical>" if sph_new
                                      else "em_tc_kernel")}
        line = {
            "metric": "EM samples/s per iteration", "value": value, "unit": "samples/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": workload_config(cfg, args),
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": traffic,
                         "kernel_path": kernel_path,
                         "kernel": ((kernel_names.get(cfg.cov_type, "?") + " (+ tc_pack_kernel, tc_reduce_kernel)")
                                    if tc_path
                                    else "topk_rows_kernel + topk_mstep_kernel + stats_reduce_kernel" if top_k
                                    else ("em_small_kernel + stats_reduce_kernel" if cfg.K <= 64
                                          else "rows_kernel + mstep_kernel + stats_reduce_kernel")),
                         "peak_source": f"{peaks['source']} bf16 {'sustained' if long_run else 'burst'}",
                         "algorithmic_flops_per_launch": flops, "launch_ms": acc_ms,
                         "hbm_frac": (n_local * cfg.B * D * torch.empty((), dtype=cfg.dtype).element_size()) /
                                     (acc_ms / 1e3) / 1e9 / peaks["hbm_gbs"]},
            "clocks": clocks,
            "gpu_launches": args.steps * launches_per_iteration(cfg, tc_path, top_k is not None),
            "e2e": e2e,
        }
        if world == 1 and not args.no_cpu:
            try:
                line["cpu_baseline"] = cpu_sample(cfg, mix, (init_means, init_cov, init_w),
                                                  args.cpu_rows or CPU_ROWS[cfg.index], approx_top_k=args.approx_top_k)
            except Exception as exc:  # report, never fake
                line["cpu_baseline"] = {"error": repr(exc)}
        print(json.dumps(line), flush=True)
    if comm:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
