"""Whole-encoder images/s on B200s, with per-kernel roofline and a CPU baseline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload: the Qwen3.5-0.8B vision encoder at 512x512
(1024 tokens, grid 32x32), fp16 weights and activations, a global batch of 64
seeded synthetic images sharded by image over N GPUs (one process per GPU,
launched by torchrun for N > 1); the embedding all-gather is the only
collective. One step = the whole encoder over the whole batch.

  value    images/s of the whole job, device-timed with CUDA events on the
           session stream, inputs resident in HBM, max over ranks.
  e2e      the same through the public API (session.Pipeline over two
           sessions): per step, the host->device copy of the step's images
           from pinned memory, the plan, the device->host copy of the
           embeddings (and the all-gather for N > 1); one step's copies
           overlap the other session's kernels.
  gather   N > 1: the embedding all-gather runs through the library's NCCL
           entry points (hexlib_b200_nccl_*, a deadline on every wait); its
           own device time per step is reported as gather_ms_per_step.
  roofline the dominant kernel (largest share of eager, op-by-op timed
           passes; each op's median of three): algorithmic FLOPs or bytes per
           launch / its mean CUDA-event duration, against MEASURED_PEAKS.json.
  cpu_baseline  the numpy oracle port (a restatement of hexlib's reference
           executor) on this host's cores, one image (rank 0, N = 1 only).

`--impl reference` times that CPU port alone on the same metric and prints
its line (rank 0; other ranks exit at once).
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
sys.path.insert(0, ROOT)

METRIC = "encoder images/s"
UNIT = "images/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--image-size", type=int, default=512)
    ap.add_argument("--batch", type=int, default=64, help="global batch (images)")
    ap.add_argument("--no-attention-fusion", action="store_true")
    ap.add_argument("--no-residual-fusion", action="store_true")
    ap.add_argument("--no-qkv-fusion", action="store_true")
    ap.add_argument("--rope", choices=("epilogue", "pass"), default="epilogue",
                    help="packed qkv path: RoPE in the qkv GEMM's epilogue, or its own pass")
    ap.add_argument("--no-patch-cast", action="store_true",
                    help="keep patchify and the cast of its rows to fp16 as two passes")
    ap.add_argument("--ln-fold", choices=("on", "off"), default="off",
                    help="fold each layernorm that feeds a GEMM into that GEMM's epilogue")
    ap.add_argument("--weights", choices=("fp16", "q4_0", "q8_0"), default="fp16",
                    help="matmul weight dtype (q4_0 is the reference model's own)")
    ap.add_argument("--gates", action="store_true",
                    help="instead of the encoder: the configuration-2 kernel gates (one GPU), "
                         "each with the reference's compiled baseline.c and the numpy "
                         "oracle timed on this host as the CPU baseline")
    ap.add_argument("--sweep", action="store_true",
                    help="instead of the encoder: the memory-bound kernel sweep (one GPU), "
                         "one JSON line per kernel and shape")
    return ap.parse_args()


def peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            m = json.load(f)
        return {"hbm": m["hbm_gbs"], "tc": m["bf16_tflops"],
                "tc_sustained": m.get("bf16_tflops_sustained", m["bf16_tflops"]),
                "src": "measured"}
    except Exception:  # noqa: BLE001
        return {"hbm": 6650.0, "tc": 1590.0, "tc_sustained": 1400.0, "src": "fallback"}


# ---- CPU baseline ----------------------------------------------------------------

def oracle_model(cfg):
    """The unfused fp16-weight plan and the weight feeds the oracle replays
    for `cfg`: for q4_0 / q8_0 weights, the same draw quantized as the plan
    stages it and dequantized to fp16 (the arithmetic the quantized GEMM
    performs), so the oracle sees exactly the weights the GPU multiplies."""
    import dataclasses

    from hexlib_b200 import feeds as F
    from hexlib_b200 import graph as G
    g = G.build_vision_encoder(cfg)
    w = F.weights(cfg, 0, g)
    if cfg.weight_dtype in ("q4_0", "q8_0"):
        from hexlib_b200 import quant
        from oracle import quant as oq
        for name, t in g.tensors.items():
            if t.const and t.dtype == cfg.weight_dtype:
                w[name] = oq.dequantize_f16(quant.quantize(w[name], t.dtype), t.shape, t.dtype)
        g = G.build_vision_encoder(dataclasses.replace(cfg, weight_dtype="fp16"))
    return G.compile_for_cuda(g), w


def cpu_port_time(cfg, n_images: int, warm: bool = True):
    """Seconds per image of the oracle port (hexlib's reference executor,
    restated) over `n_images` images, on all BLAS threads of this host; also
    the embeddings of the first image (for the parity check)."""
    from hexlib_b200 import feeds as F
    from hexlib_b200 import graph as G
    from oracle import executor
    ep, w = oracle_model(cfg)
    imgs = F.images(cfg, n_images, 1)
    if warm:  # page in numpy/BLAS on a small model
        small = G.qwen35_at(64)
        gs = G.build_vision_encoder(small)
        executor.run(G.compile_for_cuda(gs), dict(F.weights(small, 0, gs),
                                                  image=F.images(small, 1, 1)[0]))
    first = None
    t0 = time.perf_counter()
    for i in range(n_images):
        out = executor.run(ep, dict(w, image=imgs[i]))
        if i == 0:
            first = out[ep.graph.outputs[0]]
    dt = (time.perf_counter() - t0) / n_images
    threads = os.cpu_count() or 1
    try:
        import threadpoolctl
        info = threadpoolctl.threadpool_info()
        threads = max([i.get("num_threads", 1) for i in info] + [1])
    except Exception:  # noqa: BLE001
        pass
    return dt, threads, f"{n_images} image(s) at {cfg.image_size}x{cfg.image_size}", first


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from hexlib_b200 import graph as G
    cfg = G.qwen35_at(args.image_size)
    # Each image is ~20-30 s of CPU at 512^2: time at most 3 so the arm ends
    # within a few minutes whatever --steps asks for.
    n = max(1, min(args.steps, 3))
    dt, threads, sample, _ = cpu_port_time(cfg, n, warm=args.warmup > 0)
    v = 1.0 / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT,
        "n_gpus": args.gpus, "steps": n, "warmup": min(args.warmup, 1),
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "fp16 storage, fp32/fp64 compute",
        "data": "synthetic (seeded images and N(0,0.02) weights)",
        "config": {"workload": f"qwen35 vision encoder {cfg.image_size}x{cfg.image_size}, "
                               f"global batch {args.batch}, fp16", "image_size": cfg.image_size,
                   "global_batch": args.batch, "seq_len": cfg.num_tokens,
                   "parallelism": "cpu, one process"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample + ", numpy restatement of hexlib's reference "
                                            "plan executor (oracle/executor.py)"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---- clocks --------------------------------------------------------------------------

class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[tuple[float, str]] = []
        self.windows: list[tuple[float, float]] = []
        self._t0 = None

    def start(self):
        """Start sampling every 100 ms and wait for the first sample, so the
        timed windows that follow are covered from their first moment."""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.index), "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t_end = time.monotonic() + 10.0
            while not self.lines and time.monotonic() < t_end and self.proc.poll() is None:
                time.sleep(0.05)
        except Exception:  # noqa: BLE001
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))

    def begin(self):
        self._t0 = time.monotonic()

    def end(self):
        if self._t0 is not None:
            self.windows.append((self._t0, time.monotonic()))
            self._t0 = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:  # noqa: BLE001
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        # samples taken inside a timed window (one sampling period of slack at its end)
        inside = [ln for t, ln in self.lines
                  if any(a <= t <= e + 0.1 for a, e in self.windows)] if self.windows else \
                 [ln for _, ln in self.lines]
        for ln in inside:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        busy = [x for x in sm if mx and x > 0.3 * mx] or sm
        return {"sm_mhz": statistics.median(busy) if busy else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---- the B200 arm ------------------------------------------------------------------------

def op_work(plan, op_index: int, n_images: int) -> tuple[str, float, float]:
    """(bound, FLOPs, bytes) of one op of the plan over `n_images`: FLOPs of
    its contractions (2·M·N·K per GEMM, 4·T²·D per attention head) and its
    algorithmic bytes (every input read once, every output written once at
    its storage dtype). `bound` is "tensor" for the contractions, "hbm" for
    the rest."""
    from hexlib_b200 import wire
    blob = plan.blob
    hdr = wire.HDR.unpack_from(blob)
    f = wire.OP.unpack_from(blob, hdr[8] + op_index * wire.OP_SIZE)
    srcs = [s for s in f[18:24] if s != 0xFFFF]
    dsts = [d for d in f[24:28] if d != 0xFFFF]
    names = {v: k for k, v in plan.index.items()}
    P = plan.placements
    vname = plan.kinds[op_index]

    def nb(n):
        p = P[names[n]]
        return p.nbytes * (n_images if p.buffer == 1 else 1)

    nbytes = float(sum(nb(s) for s in srcs) + sum(nb(d) for d in dsts))
    if vname.startswith("matmul_epilogue"):
        a, w = P[names[srcs[0]]], P[names[srcs[1]]]
        K, N = w.shape
        return "tensor", 2.0 * a.shape[0] * n_images * N * K, nbytes
    if vname == "matmul":
        a, b = P[names[srcs[0]]], P[names[srcs[1]]]
        Bn, M, K = a.shape
        return "tensor", 2.0 * Bn * n_images * M * b.shape[2] * K, nbytes
    if vname == "attention":
        Bn, T, D = P[names[srcs[0]]].shape
        return "tensor", 4.0 * Bn * n_images * T * T * D, nbytes
    if vname == "attention_qkv":
        T, _, H, D = P[names[srcs[0]]].shape
        return "tensor", 4.0 * H * n_images * T * T * D, nbytes
    return "hbm", 0.0, nbytes


def traffic_on_record(kernel: str, image_size: int, n_images: int):
    """DRAM bytes per launch of `kernel` from the committed ncu summary
    (profiles/traffic.json), scaled to `n_images` -- only when that capture was
    taken at this image size (its bytes grow with the images, not with the
    resolution); else (None, why)."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            tr = json.load(f)
    except Exception:  # noqa: BLE001
        return None, "no ncu traffic summary on record"
    ent = tr.get(kernel)
    if ent is None:
        return None, f"no ncu capture of {kernel} on record"
    if int(ent["image_size"]) != image_size:
        return None, (f"the ncu capture of {kernel} on record is at {ent['image_size']}^2, "
                      f"not {image_size}^2")
    per_image = float(ent["bytes"]) / float(ent["images"])
    return per_image * n_images, (f"{ent['source']}; {ent['images']} images per captured "
                                  f"launch, scaled to {n_images}")


def run_b200(args) -> None:
    import numpy as np
    import torch

    from hexlib_b200 import dist as D
    from hexlib_b200 import feeds as F
    from hexlib_b200 import graph as G
    from hexlib_b200 import wholeplan
    from hexlib_b200.session import MODE_EAGER, Pipeline, Session, attention_available

    rank, local, world = D.env_rank()
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        pg = dist

    cfg = G.qwen35_at(args.image_size, weight_dtype=args.weights)
    g = G.build_vision_encoder(cfg)
    use_att = (not args.no_attention_fusion) and attention_available()
    use_qkv = use_att and not args.no_qkv_fusion
    rewrites = dict(G.DEFAULT_REWRITES)
    rewrites.update(attention=use_att, residual=not args.no_residual_fusion, qkv=use_qkv,
                    rope_epilogue=args.rope == "epilogue",
                    ln_fold=args.ln_fold == "on" and args.weights == "fp16",
                    patch_cast=not args.no_patch_cast)
    ep = G.compile_for_cuda(g, **rewrites)
    w = F.weights(cfg, 0, g)
    plan = wholeplan.build_cuda_plan(ep, w, alias=True)
    sh = D.shard(args.batch, rank, world)
    n = sh.count
    imgs = F.images(cfg, n, seed=1 + sh.start)
    host_in = torch.from_numpy(imgs).pin_memory()
    out_p = plan.placements[plan.outputs[0]]
    host_out = torch.empty((n,) + tuple(out_p.shape), dtype=torch.float16).pin_memory()

    s = Session(local)
    s.load(plan, max_images=n)
    s.write_input(plan.inputs[0], host_in, n)
    stream = torch.cuda.ExternalStream(s.stream(), device=torch.device("cuda", local))
    emb = s.device_view(plan.outputs[0], n)

    gather_events: list = []
    # The embedding all-gather (N > 1) through the library's NCCL entry points,
    # every wait bounded; one gathered [B, T/4, C_out] buffer per session.
    gatherer = D.EmbeddingGather(rank, world, local, timeout_s=120.0) if pg is not None else None
    gathered: dict = {}

    def gather_on(sess, view):
        buf = gathered.get(id(sess))
        if buf is None:
            buf = torch.empty((world * n,) + tuple(view.shape[1:]), dtype=torch.float16,
                              device=view.device)
            gathered[id(sess)] = buf
        gatherer.gather(view, buf, sess.stream())

    def step_device(timed=False):
        s.invoke(n, sync=False)
        if gatherer is not None:
            if timed:   # the all-gather's own device time, on the session stream
                g0 = torch.cuda.Event(enable_timing=True)
                g1 = torch.cuda.Event(enable_timing=True)
                g0.record(stream)
            gather_on(s, emb)
            if timed:
                g1.record(stream)
                gather_events.append((g0, g1))

    def barrier():
        if pg is not None:
            pg.barrier()
        torch.cuda.synchronize()
        s.sync()

    clocks = ClockSampler(local)
    clocks.start()
    warm = max(args.warmup, 3)
    for _ in range(warm):
        step_device()
    s.sync()

    # ---- device-timed, inputs resident ----------------------------------------------
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    clocks.begin()
    e0.record(stream)
    for _ in range(args.steps):
        step_device(timed=True)
    e1.record(stream)
    s.sync()
    e1.synchronize()
    clocks.end()
    ms = e0.elapsed_time(e1)
    t = torch.tensor([ms], device="cuda")
    if pg is not None:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    ms_max = float(t.item())
    value = args.batch * args.steps / (ms_max / 1e3)
    gather_ms = None
    if gather_events:
        t = torch.tensor([sum(a.elapsed_time(b) for a, b in gather_events) / len(gather_events)],
                         device="cuda")
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
        gather_ms = float(t.item())

    # ---- end to end through the public Pipeline API (pinned host buffers) ----------
    # Two sessions used in turn: each step uploads its images, replays the
    # plan and reads its embeddings back on its own stream, so step k+1's
    # upload overlaps step k's kernels. Every step's copies are inside the
    # timed region, which runs from before the first upload to after the
    # last read-back on every stream.
    pipe = Pipeline(plan, max_images=n, device=local, sessions=[s])
    dev = torch.device("cuda", local)
    streams = [torch.cuda.ExternalStream(x.stream(), device=dev) for x in pipe.sessions]
    views = [x.device_view(plan.outputs[0], n) for x in pipe.sessions]
    host_outs = [host_out] + [torch.empty_like(host_out).pin_memory()
                              for _ in pipe.sessions[1:]]

    def step_e2e(k):
        j = k % len(pipe.sessions)
        pipe.submit(host_in, host_outs[j])
        if gatherer is not None:
            gather_on(pipe.sessions[j], views[j])

    for k in range(len(pipe.sessions)):      # the new session captures its graph
        step_e2e(k)
    pipe.drain()
    barrier()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    clocks.begin()
    e2.record(streams[0])
    for st in streams[1:]:
        st.wait_event(e2)
    for k in range(args.steps):
        step_e2e(k)
    for st in streams[1:]:
        ev = torch.cuda.Event()
        ev.record(st)
        streams[0].wait_event(ev)
    e3.record(streams[0])
    e3.synchronize()
    clocks.end()
    clk = clocks.stop()
    pipe.drain()
    ms_e2e = e2.elapsed_time(e3)
    t = torch.tensor([ms_e2e], device="cuda")
    if pg is not None:
        pg.all_reduce(t, op=pg.ReduceOp.MAX)
    e2e = args.batch * args.steps / (float(t.item()) / 1e3)

    # ---- per-kernel roofline (eager, op-by-op timed passes) -------------------------
    # Three passes, each op's median: one pass can land on a clock dip. Each op
    # is timed alone by CUDA events around its launch, so the burst peaks of
    # MEASURED_PEAKS.json are the denominators.
    passes = [[r.cycles for r in s.invoke(n, mode=MODE_EAGER).results] for _ in range(3)]
    per_op = [sorted(v)[1] for v in zip(*passes)]
    pk = peaks()
    groups: dict[tuple, list[int]] = {}
    roof_s = 0.0          # the encoder's roofline time: sum of max(FLOPs/peak, bytes/BW)
    for i, ns in enumerate(per_op):
        bound, flops, nbytes = op_work(plan, i, n)
        roof_s += max(flops / (pk["tc"] * 1e12), nbytes / (pk["hbm"] * 1e9))
        groups.setdefault((plan.kinds[i], bound, flops, nbytes), []).append(ns)
    total_ns = sum(per_op)
    table = sorted(((sum(v), k, v) for k, v in groups.items()), reverse=True)

    def rate(bound, flops, nbytes, secs):
        return flops / secs / 1e12 if bound == "tensor" else nbytes / secs / 1e9

    dom_ns, (dname, dbound, dflops, dbytes), dlist = table[0]
    mean_s = (dom_ns / len(dlist)) / 1e9
    achieved = rate(dbound, dflops, dbytes, mean_s)
    peak, punit = (pk["tc"], "TFLOP/s") if dbound == "tensor" else (pk["hbm"], "GB/s")
    traffic, traffic_note = traffic_on_record(dname, cfg.image_size, n)

    kernels = []
    for tot, (kname, bound, flops, nbytes), lst in table:
        m = tot / len(lst) / 1e9
        a = rate(bound, flops, nbytes, m)
        kernels.append({"kernel": kname, "launches": len(lst), "share": tot / total_ns,
                        "mean_us": m * 1e6, "achieved": a,
                        "unit": "TFLOP/s" if bound == "tensor" else "GB/s",
                        "frac": a / (pk["tc"] if bound == "tensor" else pk["hbm"])})

    # ---- parity: this step's first image against the oracle (untimed) ----------------
    s.invoke(n)                                  # one more graph replay
    got0 = s.read_output(plan.outputs[0], n)[0]   # per-image tensors sit at offset x n
    cpu, parity = None, None
    if rank == 0:
        if world == 1 and os.environ.get("HEXLIB_B200_BENCH_NO_CPU") != "1":
            dt, threads, sample, ref0 = cpu_port_time(cfg, 1)
            cpu = {"value": 1.0 / dt, "unit": UNIT, "cores": threads, "kind": "port",
                   "sample": sample + " through the numpy restatement of hexlib's reference "
                                      "plan executor (oracle/executor.py)"}
        else:
            _, _, _, ref0 = cpu_port_time(cfg, 1, warm=False)
        err = float(np.abs(got0.astype(np.float64) - ref0).max() / np.abs(ref0).max())
        parity = {"status": "ok" if err < 1e-2 else "FAIL", "max_rel_err": err,
                  "bar": 1e-2, "checked": "image 0 of rank 0's shard, embeddings of the "
                                          "last graph replay against the oracle's replay "
                                          "of the unfused plan (oracle/executor.py)"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": warm, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "fp16", "data": "synthetic (seeded images, N(0,0.02) fp16 weights)",
            "config": {
                "workload": f"qwen35 vision encoder {cfg.image_size}x{cfg.image_size}, "
                            f"global batch {args.batch}, sharded by image",
                "image_size": cfg.image_size, "global_batch": args.batch,
                "seq_len": cfg.num_tokens, "parallelism": f"image-sharded x{world}",
                "weights": args.weights, "plan_ops": plan.n_ops,
                "fusions": {k: bool(v) for k, v in rewrites.items()},
                "l2": f"inputs larger than L2: each step reads {plan.const_bytes / 1e6:.0f} MB "
                      f"of consts and {host_in.numel() * 4 / 1e6:.0f} MB of images per GPU",
            },
            "e2e": {"value": e2e, "unit": UNIT,
                    "h2d_bytes_per_step": int(host_in.numel() * 4),
                    "d2h_bytes_per_step": int(host_out.numel() * 2)},
            "gpu_launches": plan.n_ops * args.steps,
            "roofline": {"kernel": dname, "bound": dbound, "achieved": achieved,
                         "peak": peak, "unit": punit, "frac": achieved / peak,
                         "peak_source": f"{pk['src']} "
                                        f"({'burst bf16' if dbound == 'tensor' else 'hbm copy'}; "
                                        f"each op timed alone)",
                         "algorithmic": dflops if dbound == "tensor" else dbytes,
                         "algorithmic_unit": "FLOP per launch" if dbound == "tensor"
                                             else "bytes per launch",
                         "traffic": traffic, "traffic_unit": "bytes per launch (dram read + write)",
                         "traffic_source": traffic_note, "share": dom_ns / total_ns,
                         "encoder_frac": (roof_s * 1e3) / (ms_max / args.steps),
                         "encoder_frac_note": "sum over the step's kernels of max(FLOPs / burst "
                                              "tensor peak, bytes / HBM copy bandwidth), over "
                                              "the device-timed ms per step"},
            "gather_ms_per_step": gather_ms,
            "parity": parity,
            "kernels": kernels[:8],
            "clocks": clk,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if gatherer is not None:
        for sess in pipe.sessions:
            gatherer.wait(sess.stream())
    pipe.close()
    s.close()
    if pg is not None:
        pg.barrier()
        gatherer.close()
        pg.destroy_process_group()


def run_sweep(args) -> None:
    """The memory-bound kernel sweep (hexlib_b200/sweep.py) on this rank's GPU;
    rank 0 prints, other ranks exit."""
    import torch

    from hexlib_b200 import dist as D
    from hexlib_b200 import sweep
    rank, local, _ = D.env_rank()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    pk = peaks()
    for row in sweep.run(pk["hbm"]):
        row["peak_gbs"] = pk["hbm"]
        row["peak_source"] = f"{pk['src']} (hbm copy)"
        print(json.dumps(row), flush=True)


def _gate_cpu(case):
    """CPU baselines of one gate: the reference's own scalar kernel
    (kernels/<kernel>/baseline.c, compiled into oracle/_ref; one core) and the
    numpy restatement (oracle/ops.py), median seconds of 5 (or 3) runs. The
    matmul_epilogue baseline.c takes q4_0 weights only (its signature in
    kernel_api.h), so it is timed with the weight quantized."""
    import ctypes
    import time

    import numpy as np

    from hexlib_b200 import quant
    from oracle import cref, ops
    r = np.random.default_rng(1)
    R, C, k = case.rows, case.width, case.kind
    F = ctypes.c_float

    def f16(*shape):
        return r.standard_normal(shape).astype(np.float16)

    ref, numpy_fn = None, None
    if k == "matmul_epilogue":
        M, N, K = R, C, case.depth
        a, w = f16(M, K), (0.02 * r.standard_normal((K, N))).astype(np.float32)
        b = (0.02 * r.standard_normal(N)).astype(np.float32)
        raw = np.frombuffer(quant.quantize_q4_0(w), np.uint8).copy()
        y = np.empty((M, N), np.float16)
        ref = lambda: cref.call("matmul_epilogue_fp16", a, raw, b, y, M, K, N, 1)  # noqa: E731
        numpy_fn = lambda: ops.matmul_epilogue(  # noqa: E731
            (a.astype(np.float32), w.astype(np.float16).astype(np.float32), b),
            {"act": "gelu_tanh"})
    elif k in ("softmax", "layernorm", "rmsnorm", "add", "scale"):
        x, y = f16(R, C), np.empty((R, C), np.float16)
        if k == "softmax":
            ref = lambda: cref.call("softmax_fp16", x, y, R, C)  # noqa: E731
            numpy_fn = lambda: ops.softmax((x,), {"axis": -1})  # noqa: E731
        elif k == "layernorm":
            w1 = (1 + 0.02 * r.standard_normal(C)).astype(np.float32)
            b1 = (0.02 * r.standard_normal(C)).astype(np.float32)
            ref = lambda: cref.call("layernorm_fp16", x, w1, b1, y, R, C, F(1e-6))  # noqa: E731
            numpy_fn = lambda: ops.layernorm((x, w1, b1), {"eps": 1e-6})  # noqa: E731
        elif k == "rmsnorm":
            g1 = f16(C)
            ref = lambda: cref.call("rmsnorm_fp16", x, g1, y, R, C, F(1e-6))  # noqa: E731
            numpy_fn = lambda: ops.rmsnorm((x, g1), {"eps": 1e-6})  # noqa: E731
        elif k == "add":
            x2 = f16(R, C)
            ref = lambda: cref.call("add_fp16", x, x2, y, R * C)  # noqa: E731
            numpy_fn = lambda: ops.add((x, x2), {})  # noqa: E731
        else:
            ref = lambda: cref.call("scale_fp16", x, y, R * C, F(0.125))  # noqa: E731
            numpy_fn = lambda: ops.scale((x,), {"factor": 0.125})  # noqa: E731
    elif k == "cast":
        x, y = r.standard_normal((R, C)).astype(np.float32), np.empty((R, C), np.float16)
        ref = lambda: cref.call("cast_f32_f16", x, y, R * C)  # noqa: E731
        numpy_fn = lambda: ops.cast((x,), {"dtype": "fp16"})  # noqa: E731
    elif k in ("rope_2d", "transpose_th", "transpose_hd"):
        H, D = case.heads, 64
        if k == "rope_2d":
            x, y = f16(R, H, D), np.empty((R, H, D), np.float16)
            ang = r.uniform(0, 6.283, (R, D)).astype(np.float32)
            cs, sn = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
            ref = lambda: cref.call("rope_2d_fp16", x, cs, sn, y, R, H, D)  # noqa: E731
            numpy_fn = lambda: ops.rope_2d((x, cs, sn), {})  # noqa: E731
        elif k == "transpose_th":
            x, y = f16(R, H, D), np.empty((H, R, D), np.float16)
            ref = lambda: cref.call("transpose_th_fp16", x, y, R, H, D)  # noqa: E731
            numpy_fn = lambda: np.ascontiguousarray(  # noqa: E731
                ops.transpose((x,), {"perm": (1, 0, 2)})[0])
        else:
            x, y = f16(H, R, D), np.empty((H, D, R), np.float16)
            ref = lambda: cref.call("transpose_hd_fp16", x, y, H, R, D)  # noqa: E731
            numpy_fn = lambda: np.ascontiguousarray(  # noqa: E731
                ops.transpose((x,), {"perm": (0, 2, 1)})[0])

    def med(fn):
        # median of 5 runs (of 3 when one run takes over half a second)
        ts = []
        for i in range(5):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
            if i == 2 and min(ts) > 0.5:
                break
        return sorted(ts)[len(ts) // 2]

    out = {}
    if ref is not None and cref.available():
        out["baseline_c_us"] = round(med(ref) * 1e6, 1)
    if numpy_fn is not None:
        out["numpy_oracle_us"] = round(med(numpy_fn) * 1e6, 1)
    return out


def run_gates(args) -> None:
    """The configuration-2 kernel gates on this rank's GPU (rank 0 prints)."""
    import torch

    from hexlib_b200 import dist as D
    from hexlib_b200 import sweep
    rank, local, _ = D.env_rank()
    if rank != 0:
        return
    torch.cuda.set_device(local)
    pk = peaks()
    for cs in sweep.GATES:
        t = sweep.time_case(cs, reps=20)
        row = {"gate": cs.kind, "shape": cs.label(), "us": round(t * 1e6, 2)}
        if cs.flops:
            tf = cs.flops / t / 1e12
            row.update({"bound": "tensor", "achieved": round(tf, 1), "unit": "TFLOP/s",
                        "peak": pk["tc"], "frac": round(tf / pk["tc"], 4)})
        else:
            gbs = cs.bytes / t / 1e9
            row.update({"bound": "hbm", "achieved": round(gbs, 1), "unit": "GB/s",
                        "peak": pk["hbm"], "frac": round(gbs / pk["hbm"], 4)})
        row["peak_source"] = pk["src"]
        row["cpu_baseline"] = dict(_gate_cpu(cs), cores=1,
                                   kind="reference baseline.c and the numpy port")
        print(json.dumps(row), flush=True)


def main():
    args = parse()
    if args.gates:
        run_gates(args)
    elif args.sweep:
        run_sweep(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
