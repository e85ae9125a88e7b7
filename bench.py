#!/usr/bin/env python
"""Benchmark of the Holmes hot path on B200.

Default workload (``--workload layer``, BASELINE config 3; one "step"): one encrypted Llama-3-8B decoder layer, a
128-token prefill on one B200 -- the reference's own one-layer application (``llama3fhe`` TransformerLayer.forward /
graph.prefill.evaluate with the synthetic preset of its ``run_layer0.py``, installed unchanged in baseline/_ref) with
every FHE operation on libholmes_cuda through the ``easyfhe`` compatibility layer: QKV / W_O / MLP projections (BSGS
linear), attention with its softmax, RMSNorm and SiLU polynomials, and the bootstraps the reference's schedule places,
at the production CKKS parameters (N = 2^16, 38 limbs of 59/60-bit primes, dnum 5).  ``value`` = device seconds per
layer with the input ciphertexts resident in HBM; ``e2e`` = the same with the inputs copied from pinned host memory
and the outputs copied back inside every timed step.  Under torchrun every rank runs its own replica (the reference's
one-layer graph is a single-process program): replicas only.  Without baseline/_ref the default falls back to the
linear workload below.

``--workload linear``: one encrypted 4096 x 4096 complex weight page applied to the 16 input ciphertexts of a
128-token prefill -- the QKV projection of one Llama-3-8B layer in the reference's feature-major layout
(llama3fhe/operators/linear/prefill/qkv_kernel.py:678-940) -- through ``LinearOperator.apply`` with the production
schedule (baby 64, 8 chunks of 8 giants) at the linear entry level of 13 limbs; every step rebuilds the baby basis,
re-encodes all 4096 diagonal rows online (pack -> special FFT -> round -> NTT) and rescales.  Multi-GPU
(``--parallelism chunk``): rank r key-switches 1 / W of the baby rotations, an NCCL all-gather completes the basis,
each rank MACs its 8 / W BSGS chunks, and a modular reduce-scatter delivers each rank its token shard;
``--parallelism token`` gives each rank 16 / W inputs end to end with no data-path collective.

``--impl reference`` times the CPU restatement of the same path (``oracle/``) on the host cores, on a bounded
sample scaled to the workload.  EasyFHE, the reference's engine, is not distributed with the reference and
cannot run here.
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

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "encrypted Llama-3-8B prefill-128 linear page latency (QKV page: 16 ciphertexts x 4096x4096)"
UNIT = "s"
LOG_N, DEPTH, DNUM, DCRT, FIRST = 16, 37, 5, 59, 60
CUR_LIMBS = 13
DIM, LANES, INPUTS = 4096, 8, 16


def measured_traffic(family: str, algorithmic_bytes: int):
    """DRAM bytes per launch of a kernel family: the committed ncu capture (profiles/traffic.txt: measured bytes and
    algorithmic bytes of the captured launch) scaled by this run's algorithmic bytes per launch (the family's traffic
    grows in proportion to the items and limbs it processes), or None."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.txt"), encoding="utf-8") as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 3 and not line.startswith("#") and parts[0] == family:
                    return int(round(int(parts[1]) / int(parts[2]) * int(algorithmic_bytes)))
    except (OSError, ValueError, ZeroDivisionError):
        pass
    return None


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json"), encoding="utf-8") as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


# ----------------------------------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int) -> None:
        self.device_index = device_index
        self.lines: list[str] = []
        self.proc = None
        self.thread = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def ready(self, timeout: float = 5.0) -> None:
        """Wait for nvidia-smi's first sample, then keep only samples from here on (the timed region starts
        right after this call)."""
        t0 = time.time()
        while self.proc is not None and not self.lines and time.time() - t0 < timeout:
            time.sleep(0.02)
        self.first = len(self.lines)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        # samples from the timed region; when it is shorter than one sampling period, the sample at its start
        first = getattr(self, "first", 0)
        window = self.lines[first:] or self.lines[max(0, first - 1):first]
        for line in window:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------------------------------- workload
def hadamard_rotation(dim: int, seed: int) -> np.ndarray:
    """Seeded +-1 diagonal times the normalised Walsh-Hadamard matrix (QuaRot-style rotation)."""
    from scipy.linalg import hadamard

    rng = np.random.default_rng(seed)
    signs = rng.choice([-1.0, 1.0], size=dim)
    return (hadamard(dim).astype(np.float64) / np.sqrt(dim)) * signs[None, :]


def make_weight(seed: int = 1) -> np.ndarray:
    rng = np.random.default_rng(seed)
    w = rng.normal(scale=0.02, size=(DIM, DIM)) + 1j * rng.normal(scale=0.02, size=(DIM, DIM))
    return w @ hadamard_rotation(DIM, seed + 1)


def make_inputs(n_inputs: int, seed: int = 0) -> np.ndarray:
    """FM-packed complex carriers: slot(d, t) = d * 8 + t, z = x_even + i x_odd (and conjugates)."""
    rng = np.random.default_rng(seed)
    x = rng.normal(size=(n_inputs, LANES, DIM)) + 1j * rng.normal(size=(n_inputs, LANES, DIM))
    return np.ascontiguousarray(x.transpose(0, 2, 1).reshape(n_inputs, DIM * LANES))


def spec_for(cur_limbs: int):
    from holmes_b200 import fhe as F
    from holmes_b200 import linear as LN

    cfg = LN.PRODUCTION
    rots = cfg.rotation_keys(DIM, LANES)
    return F.CKKSContextSpec(depth=DEPTH, log_n=LOG_N, dnum=DNUM, dcrt_bits=DCRT, first_mod=FIRST, special_bits=60,
                             hamming_weight=192, seed=0, rotations=tuple(rots), auto_load_keys=False,
                             rotation_key_limb_limits={int(r): cur_limbs for r in rots}), cfg, rots


def run_engine(args) -> None:
    import torch
    import torch.distributed as dist

    from holmes_b200 import _lib
    from holmes_b200 import fhe as F
    from holmes_b200 import linear as LN

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    from holmes_b200 import collectives as C

    n_inputs = args.inputs
    mine = list(C.token_shard(n_inputs, world, rank))
    chunked = args.parallelism == "chunk" and world > 1
    cur = args.limbs
    spec, cfg, rots = spec_for(cur)
    client, ctx = F.generate_client_context(spec, f"cuda:{local}")
    session = LN.Session(client, ctx)
    ctx.generate_rotation_keys(rots, cur)
    level = ctx.L - cur
    weight = make_weight()
    carriers = make_inputs(n_inputs)
    # chunk sharding: every rank holds all inputs and MACs its BSGS chunks; token sharding: its own inputs
    held = list(range(n_inputs)) if chunked else mine
    cts = [session.encrypt(carriers[i], level=level, counter=i) for i in held]
    # chunk sharding also splits the baby key switches over the ranks and all-gathers the basis
    op = LN.LinearOperator(crypto_context=session, token_lanes=LANES, config=cfg,
                           baby_shard=(rank, world, None) if chunked else None)
    lw = LN.LinearWeight(weight, dtype=np.complex128, crypto_context=session)
    lw.prepare(cfg)
    my_chunks = C.chunk_shard(len(op.layout(DIM).chunks), world, rank)
    torch.cuda.synchronize()

    def step():
        op.clear_baby_cache()
        return page(op, cts, lw)

    def page(op_, cts_, lw_):
        if not chunked:
            outs, _ = op_.apply(cts_, lw_)
            return outs
        parts, _ = op_.apply(cts_, lw_, chunk_indices=my_chunks, rescale=False)
        p0 = torch.cat([p.cv[0] for p in parts])
        p1 = torch.cat([p.cv[1] for p in parts])
        s0 = C.modular_reduce_scatter(ctx, p0, world)
        s1 = C.modular_reduce_scatter(ctx, p1, world)
        batch = F.Cipher([s0, s1], parts[0].state, parts[0].slots, False, len(mine), ctx)
        res = F.rescale(batch, ctx)
        return [res.cipher_like([res.cv[0][i:i + 1], res.cv[1][i:i + 1]], batch_size=1) for i in range(len(mine))]

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    sampler.ready()
    if world > 1:
        dist.barrier()
    count0 = _lib.ctypes.c_ulonglong()
    _lib.call("holmes_launch_count", _lib.ctypes.byref(count0))
    F.OPTIMER.reset()
    F.OPTIMER.enabled = True
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("timed")
    start.record()
    for _ in range(args.steps):
        outs = step()
    end.record()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    F.OPTIMER.enabled = False
    count1 = _lib.ctypes.c_ulonglong()
    _lib.call("holmes_launch_count", _lib.ctypes.byref(count1))
    clocks = sampler.stop()
    ms = start.elapsed_time(end) / args.steps
    ops = F.OPTIMER.summary()
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()

    # ---- end to end through the public API: inputs and weight from pinned host memory, outputs back
    host_in = [torch.stack([c.cv[0][0], c.cv[1][0]]).cpu().pin_memory() for c in cts]
    host_w = torch.from_numpy(np.ascontiguousarray(weight)).pin_memory()
    out_bytes = 0

    def e2e_step():
        nonlocal out_bytes
        dev_in = []
        for h in host_in:
            d = h.to(ctx.device, non_blocking=True)
            dev_in.append(F.Cipher([d[0:1], d[1:2]], cts[0].state, cts[0].slots, False, 1, ctx))
        # the pinned page goes to LinearWeight as is: it uploads it on a side stream behind the baby rotations
        with LN.LinearWeight(host_w, dtype=np.complex128, crypto_context=session) as lw2:
            with LN.LinearOperator(crypto_context=session, token_lanes=LANES, config=cfg,
                                   baby_shard=(rank, world, None) if chunked else None) as op2:
                res = page(op2, dev_in, lw2)
        back = [torch.stack([r.cv[0][0], r.cv[1][0]]).to("cpu", non_blocking=True) for r in res]
        out_bytes = sum(b.numel() * 8 for b in back)
        return back

    e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    if world > 1:
        t = torch.tensor([e2e_ms], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    in_bytes = sum(h.numel() * 8 for h in host_in) + host_w.numel() * 16

    # ---- a parity spot check of this run's output (decrypted vs NumPy), outside all timing
    check = None
    if rank == 0 and args.check:
        dec = session.decrypt(outs[0]).reshape(DIM, LANES)
        x = carriers[mine[0]].reshape(DIM, LANES)
        check = float(np.abs(dec - weight @ x).max())

    if rank == 0:
        hbm, kind = peaks()
        dominant = max(ops.items(), key=lambda kv: kv[1]["ms"]) if ops else None
        roofline = None
        if dominant:
            name, d = dominant
            per_launch_s = d["ms"] / 1e3 / d["launches"]
            achieved = d["bytes"] / d["launches"] / per_launch_s / 1e9
            roofline = {"bound": "hbm", "kernel": name, "achieved": round(achieved, 1), "peak": hbm,
                        "peak_kind": kind, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                        "traffic": measured_traffic(name, d["bytes"] // d["launches"]),
                        "algorithmic_bytes_per_launch": d["bytes"] // d["launches"],
                        "avg_launch_ms": round(d["ms"] / d["launches"], 4),
                        "share_of_step": round(d["ms"] / args.steps / ms, 4)}
        cpu = None
        if args.cpu_baseline and world == 1:
            cpu = cpu_baseline(rows=args.cpu_rows)
        line = {
            "metric": METRIC, "value": round(ms / 1e3, 5), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 3), "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "u64 (RNS residues, 59/60-bit primes)", "data": "synthetic (seeded)",
            "config": {"workload": f"QKV-shaped linear page: {n_inputs} ciphertexts x one 4096x4096 complex page, "
                                   f"N=2^16, {cur}/{DEPTH + 1} limbs, dnum {DNUM} (alpha {ctx.alpha}, K {ctx.K}), "
                                   f"baby 64, 8 chunks x 8 giants, lanes 8, rescale",
                       "parallelism": (f"chunk-sharded x{world} + baby all-gather + modular reduce-scatter" if chunked
                                       else f"token-sharded x{world}"), "inputs_per_rank": len(mine),
                       "l2": "working set (plaintext chunks 3.4 GB, baby basis 13.6 GB) >> 126 MB L2",
                       "keys": f"{len(rots)} rotation keys capped at {cur} limbs"},
            "roofline": roofline, "kernels": {k: {"launches": v["launches"], "ms_per_step": round(v["ms"] / args.steps, 3)}
                                              for k, v in ops.items()},
            "cpu_baseline": cpu, "clocks": clocks,
            "e2e": {"value": round(e2e_ms / 1e3, 5), "unit": UNIT, "h2d_bytes_per_step": in_bytes,
                    "d2h_bytes_per_step": out_bytes},
            "gpu_launches": int(count1.value - count0.value) // args.steps,
            "parity_check_max_abs_err": check,
        }
        print(json.dumps(line), flush=True)
    lw.close()
    op.close()
    ctx.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ----------------------------------------------------------------------------------------------------- CPU leg
def cpu_baseline(rows: int = 128, hoisted: int = 6, rotations: int = 3) -> dict:
    """Time the CPU restatement (oracle/) on a bounded sample of the page and scale it to one page.

    Sample (about 10 s on 16 cores): ``rows`` diagonal rows encoded at 13 limbs, their MAC against one input's
    babies, one ModUp, ``hoisted`` hoisted baby key switches and ``rotations`` Horner giant key switches; the page
    is 4096 rows x 16 inputs, 16 x 63 baby and 16 x (8 x 7 + 7) giant / alignment key switches.
    """
    os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))
    from oracle.oracle import Oracle, OracleParams

    cores = int(os.environ["OMP_NUM_THREADS"])
    pr = OracleParams(log_n=LOG_N, limbs=DEPTH + 1, dnum=DNUM, dcrt_bits=DCRT, first_mod_bits=FIRST, special_bits=60,
                      hamming=192, seed=0)
    o = Oracle(pr)
    cur = CUR_LIMBS
    rng = np.random.default_rng(0)
    z = rng.normal(scale=0.02, size=(rows, pr.n // 2)) + 1j * rng.normal(scale=0.02, size=(rows, pr.n // 2))
    t0 = time.perf_counter()
    pts = np.stack([o.encode(z[r], cur) for r in range(rows)])
    t_enc = (time.perf_counter() - t0) / rows
    ct = o.encrypt(rng.normal(size=pr.n // 2), cur, counter=0)
    babies = [(ct[0], ct[1])] * rows
    t0 = time.perf_counter()
    o.bsgs_mac(pts, babies, 1)
    t_mac = (time.perf_counter() - t0) / rows
    baby_offsets = [8 * (b + 1) for b in range(hoisted)]
    for r in baby_offsets + [512]:
        o.rotation_key(o.galois(r), cap=cur)
    t0 = time.perf_counter()
    digits = o.modup(ct[1])
    t_modup = time.perf_counter() - t0
    t0 = time.perf_counter()
    for r in baby_offsets:
        o.rotate(ct, r, digits=digits, cap=cur)
    t_hoisted = (time.perf_counter() - t0) / hoisted
    t0 = time.perf_counter()
    acc = ct
    for _ in range(rotations):
        acc = o.rotate(acc, 512, cap=cur)
    t_rot = (time.perf_counter() - t0) / rotations
    page = (4096 * t_enc + 4096 * INPUTS * t_mac + INPUTS * (t_modup + 63 * t_hoisted)
            + INPUTS * (8 * 7 + 7) * t_rot)
    return {"value": round(page, 2), "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{rows} rows encoded + MAC'd at N=2^16 / 13 limbs, 1 ModUp, {hoisted} hoisted + {rotations} "
                      "full key switches; scaled to 4096 rows x 16 inputs, 16x63 baby and 16x63 giant/alignment key "
                      "switches",
            "per_op_s": {"encode_row": round(t_enc, 4), "mac_row_input": round(t_mac, 4), "modup": round(t_modup, 4),
                         "hoisted_ks": round(t_hoisted, 4), "rotation": round(t_rot, 4)}}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    for _ in range(args.warmup):
        cpu_baseline(rows=4, hoisted=1, rotations=1)   # untimed: pages in the oracle and its tables
    vals = []
    cpu = None
    for _ in range(max(1, args.steps)):
        cpu = cpu_baseline()
        vals.append(cpu["value"])
    v = statistics.median(vals)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "u64 (RNS residues)", "data": "synthetic (seeded)",
            "config": {"workload": "QKV-shaped linear page (CPU restatement of the reference path; EasyFHE itself "
                                   "is not distributed and cannot run here)"},
            "cpu_baseline": {**cpu, "value": v},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_kernel(args) -> None:
    """One bench-shaped launch of one kernel family (N = 2^16, 13 limbs, 16 ciphertexts), after one warm-up
    launch, for profiler captures: ``mac`` (one chunk: 8 giants x 64 babies), ``keyswitch`` (the key switch of
    one baby rotation: inner products, P-limb iNTT, P -> Q conversion, Q-limb NTT), ``modup``, ``ntt`` (forward NTT of 16 x 13 polynomials), ``encode`` (one chunk's 512 rows).
    ``--inputs`` / ``--limbs`` shrink the case (multi-pass captures want a few GB on the device); at the bench
    shape memory on the device stays below 20 GB."""
    import torch

    from holmes_b200 import _lib as L
    from holmes_b200 import fhe as F

    spec, _, _ = spec_for(CUR_LIMBS)
    _, ctx = F.generate_client_context(spec)
    N, cur, I = ctx.N, int(args.limbs), int(args.inputs)

    def rand(items, limbs):
        out = torch.empty((items, limbs, N), dtype=torch.uint64, device=ctx.device)
        for li in range(limbs):
            r = torch.randint(0, 2 ** 62, (items, N), device=ctx.device, dtype=torch.int64)
            out[:, li] = (r % ctx.moduli[li]).to(torch.uint64)
        return out

    if args.kernel == "mac":
        nb, G = 64, 8
        pts = rand(G * nb, cur)
        bab = rand(2 * nb * I, cur).reshape(2, nb, I, cur, N)
        res = torch.empty((2, G, I, cur, N), dtype=torch.uint64, device=ctx.device)
        c0s = L.ptr_array([bab[0, :, i].data_ptr() for i in range(I)])
        c1s = L.ptr_array([bab[1, :, i].data_ptr() for i in range(I)])

        def fn():
            L.call("holmes_bsgs_mac", ctx.handle, res.data_ptr(), c0s, c1s, I * cur * N, nb, I, pts.data_ptr(),
                   cur * N, G, cur, 0)
    elif args.kernel in ("keyswitch", "modup"):
        c0, c1 = rand(I, cur), rand(I, cur)
        o0, o1 = torch.empty_like(c0), torch.empty_like(c1)
        g = ctx.galois(LANES)
        key = ctx.switch_key(g, cur)
        digits, dig_item = F._modup(ctx, c1, cur, I)

        def fn():
            if args.kernel == "modup":
                F._modup(ctx, c1, cur, I)
            else:
                F._keyswitch(ctx, digits, dig_item, cur, g, key, c0, None, F._item_stride(c0), o0, o1, I)
    elif args.kernel == "ntt":
        x = rand(I, cur)

        def fn():
            L.call("holmes_ntt", ctx.handle, x.data_ptr(), I, cur, cur * N, 0, 0, 0)
    elif args.kernel == "encode":
        rows = torch.randn((512, ctx.max_slots), dtype=torch.complex128, device=ctx.device) * 0.02
        mid = F.fft_special_inv_rows(ctx, rows, ctx.max_slots)

        def fn():
            F.encode_rows(ctx, mid, cur, ctx.scale, ctx.max_slots, already_transformed=True)
    else:
        raise SystemExit(f"unknown kernel family {args.kernel}")
    fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    fn()
    b.record()
    torch.cuda.synchronize()
    print(json.dumps({"kernel": args.kernel, "ms": round(a.elapsed_time(b), 3)}), flush=True)
    ctx.close()


def _ref_kernel_lib(name: str):
    """The reference's own in-tree CUDA kernel library (bench/cmp/kernels/*.cu compiled unchanged for sm_100a by
    ``make -C oracle ref``): the bar the engine's kernels are measured against.  None when not built."""
    import ctypes

    path = os.path.join(ROOT, "oracle", "_ref", name)
    return ctypes.CDLL(path) if os.path.exists(path) else None


def _root_tables_from_engine(ctx, limbs: int):
    """power_of_roots / power_of_roots_shoup in the reference's layout ([limbs][N], psi^bitrev(k)) for the engine's
    own primes.  psi is read back from the engine: the NTT of the monomial X has psi^(2 bitrev(0) + 1) = psi in
    word 0."""
    import torch

    from holmes_b200 import _lib as L

    N = ctx.N
    x = torch.zeros((1, limbs, N), dtype=torch.uint64, device=ctx.device)
    x[0, :, 1] = 1
    L.call("holmes_ntt", ctx.handle, x.data_ptr(), 1, limbs, limbs * N, 0, 0, 0)
    psis = [int(v) for v in x[0, :, 0].cpu().numpy()]
    bits = ctx.logN
    rev = np.array([int(format(k, f"0{bits}b")[::-1], 2) for k in range(N)])
    roots = np.empty((limbs, N), dtype=np.uint64)
    shoup = np.empty((limbs, N), dtype=np.uint64)
    for li in range(limbs):
        q, psi = ctx.moduli[li], psis[li]
        pw = [1] * N
        for k in range(1, N):
            pw[k] = pw[k - 1] * psi % q
        r = [pw[int(j)] for j in rev]
        roots[li] = np.array(r, dtype=np.uint64)
        shoup[li] = np.array([(v << 64) // q for v in r], dtype=np.uint64)
    return roots, shoup


def run_vs_ref(args) -> None:
    """The engine's kernels against the reference's own in-tree kernels on the same B200, same inputs, bench shape
    (N = 2^16, 13 limbs of the production chain):

    * ``--kernel mac``: one BSGS chunk (8 giants x 64 babies, 16 inputs) -- the reference's ``holmes_mac_multi`` at its
      production tile ``ti = 10108`` (lazy 1 x 8, bench/cmp/holmes_multi_mac.py:57-58; kernel
      bench/cmp/kernels/holmes_mac.cu:196-274) against the engine's ``holmes_bsgs_mac`` (``k_bsgs_mac3``);
    * ``--kernel encode``: encode stage 2 of one chunk's 512 rows (llround, per-limb reduction, NTT) -- the reference's
      ``holmes_encode_stage2`` with its default launch (bench/cmp/holmes_fast_stage2.py:43-49; kernels
      bench/cmp/kernels/holmes_encode.cu:115-285) against the engine's ``holmes_encode_fft`` on the same doubles.

    Both outputs are compared word for word before timing; each side is timed with CUDA events over ``--steps``
    launches after ``--warmup`` launches, the clocks sampled during the timed launches."""
    import ctypes

    import torch

    from holmes_b200 import _lib as L
    from holmes_b200 import fhe as F

    spec, _, _ = spec_for(CUR_LIMBS)
    _, ctx = F.generate_client_context(spec)
    N, cur, I = ctx.N, int(args.limbs), int(args.inputs)
    gen = torch.Generator(device=ctx.device).manual_seed(0)

    def rand(items, limbs):
        out = torch.empty((items, limbs, N), dtype=torch.uint64, device=ctx.device)
        for li in range(limbs):
            r = torch.randint(0, 2 ** 62, (items, N), device=ctx.device, dtype=torch.int64, generator=gen)
            out[:, li] = (r % ctx.moduli[li]).to(torch.uint64)
        return out

    p, i32, ll, d = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_double
    if args.kernel == "mac":
        lib = _ref_kernel_lib("libholmes_mac_ref.so")
        if lib is None:
            raise SystemExit("oracle/_ref/libholmes_mac_ref.so is not built (make -C oracle ref)")
        lib.holmes_mac_multi.argtypes = [p, p, p, ll, i32, i32, p, ll, i32, i32, i32, p, p, p, p]
        lib.holmes_mac_multi.restype = i32
        nb, G = 64, 8
        pts = rand(G * nb, cur)
        bab = rand(2 * nb * I, cur).reshape(2, nb, I, cur, N)
        c0s = L.ptr_array([bab[0, :, i].data_ptr() for i in range(I)])
        c1s = L.ptr_array([bab[1, :, i].data_ptr() for i in range(I)])
        res_ref = torch.empty((2, G, I, cur, N), dtype=torch.uint64, device=ctx.device)
        res_eng = torch.empty_like(res_ref)
        tabs = (ctx.primes.data_ptr(), ctx.barret_ratio.data_ptr(), ctx.barret_k.data_ptr())

        def ref():
            rc = lib.holmes_mac_multi(res_ref.data_ptr(), c0s, c1s, I * cur * N, nb, I, pts.data_ptr(), cur * N, G,
                                      10108, cur, *tabs, None)
            if rc:
                raise RuntimeError(f"reference holmes_mac_multi returned {rc}")

        def eng():
            L.call("holmes_bsgs_mac", ctx.handle, res_eng.data_ptr(), c0s, c1s, I * cur * N, nb, I, pts.data_ptr(),
                   cur * N, G, cur, 0)
        nbytes = (G * nb * cur + I * nb * 2 * cur + 2 * G * I * cur) * N * 8
        outs = (res_ref, res_eng)
        what = "BSGS MAC chunk: 8 giants x 64 babies x 16 inputs, 13 limbs"
    elif args.kernel == "encode":
        lib = _ref_kernel_lib("libholmes_encode_ref.so")
        if lib is None:
            raise SystemExit("oracle/_ref/libholmes_encode_ref.so is not built (make -C oracle ref)")
        lib.holmes_encode_stage2.argtypes = [p, p, ll, i32, d, i32, p, p, p, p, p, p, p, i32, i32, i32]
        lib.holmes_encode_stage2.restype = i32
        rows = 512
        z = torch.randn((rows, ctx.max_slots), dtype=torch.complex128, device=ctx.device, generator=gen) * 0.02
        mid = F.fft_special_inv_rows(ctx, z, ctx.max_slots)
        zr = torch.view_as_real(mid).contiguous()            # the stage-1 doubles: [rows][N/2][re, im]
        roots, shoup = _root_tables_from_engine(ctx, cur)
        k_max64 = 9223372036854775295                         # Encode.cu MAX_64BIT_VALUE (holmes_encode.cu:14)
        diffs = torch.tensor([k_max64 % q for q in ctx.moduli[:cur]], dtype=torch.uint64, device=ctx.device)
        rt = torch.from_numpy(roots).to(ctx.device)
        st = torch.from_numpy(shoup).to(ctx.device)
        out_ref = torch.empty((rows, cur, N), dtype=torch.uint64, device=ctx.device)
        out_eng = torch.empty_like(out_ref)
        flag = torch.zeros(1, dtype=torch.int32, device=ctx.device)
        scale = float(ctx.scale)

        def ref():
            rc = lib.holmes_encode_stage2(out_ref.data_ptr(), zr.data_ptr(), N, rows, scale, cur,
                                          ctx.primes.data_ptr(), diffs.data_ptr(), ctx.barret_ratio.data_ptr(),
                                          ctx.barret_k.data_ptr(), rt.data_ptr(), st.data_ptr(),
                                          torch.cuda.current_stream().cuda_stream, 0, 3, 0)
            if rc:
                raise RuntimeError(f"reference holmes_encode_stage2 returned {rc}")

        def eng():
            L.call("holmes_encode_fft", ctx.handle, zr.data_ptr(), N, rows, ctx.max_slots, scale, cur,
                   out_eng.data_ptr(), cur * N, flag.data_ptr(), 0)
        nbytes = rows * (N * 8 + cur * N * 8)
        outs = (out_ref, out_eng)
        what = "encode stage 2: 512 rows (one BSGS chunk), 13 limbs"
    else:
        raise SystemExit("--vs-ref covers --kernel mac and --kernel encode")
    ref()
    eng()
    torch.cuda.synchronize()
    if not torch.equal(outs[0], outs[1]):
        raise SystemExit(f"{args.kernel}: engine and reference outputs differ")

    def timed(fn):
        for _ in range(max(1, args.warmup)):
            fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(max(1, args.steps)):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / max(1, args.steps)

    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    clocks.ready()
    t_ref = timed(ref)
    t_eng = timed(eng)
    ck = clocks.stop()
    peak, kind = peaks()
    print(json.dumps({"kernel": args.kernel, "vs_ref": what, "bit_identical": True, "ref_ms": round(t_ref, 4),
                      "engine_ms": round(t_eng, 4), "speedup": round(t_ref / t_eng, 3),
                      "algorithmic_bytes": nbytes, "engine_hbm_frac": round(nbytes / (t_eng * 1e-3) / 1e9 / peak, 4),
                      "ref_hbm_frac": round(nbytes / (t_ref * 1e-3) / 1e9 / peak, 4), "peak_gbs": peak,
                      "peak_kind": kind, "clocks": ck}), flush=True)
    ctx.close()


LAYER_METRIC = "encrypted Llama-3-8B prefill-128 one-decoder-layer latency (1 B200)"


def _reference_application():
    """Put the reference's own llama3fhe (installed unchanged in baseline/_ref by tests/install_reference.py) on the
    path with this engine registered as its ``easyfhe``."""
    ref = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref, "llama3fhe")):
        raise SystemExit("--workload layer drives the reference's own layer graph on this engine; install the "
                         "reference first: python tests/install_reference.py <checkout of the reference>")
    if ref not in sys.path:
        sys.path.insert(0, ref)
    from holmes_b200 import easyfhe_compat

    easyfhe_compat.install()


class _LayerSetup:
    """BASELINE config 3 through the reference's own one-layer application path (the synthetic preset of its
    ``run_layer0.py``: ``llama3fhe/application/runner.py:158-470``): Llama-3-8B geometry (hidden 4096, 32 query / 8
    KV heads of 128, MLP 14336), 128 prefill tokens feature-major packed into 16 ciphertexts at N = 2^16, the
    production chain (38 limbs, dnum 5), the reference's polynomial tables and its layer schedule, RoPE theta 5e5,
    bootstraps where the schedule places them.  Everything above the engine -- layer graph, operators, attention,
    bootstrap policy -- is the reference's code, unchanged; every FHE operation runs on libholmes_cuda."""

    def __init__(self, seed: int) -> None:
        _reference_application()
        import numpy as _np

        from llama3fhe import Llama3CKKSConfig
        from llama3fhe.application.approx_config import ApproximationConfig
        from llama3fhe.application.args import build_parser, resolve_poly_paths
        from llama3fhe.application.inputs import _synthetic_inputs
        from llama3fhe.application.layer_stream import DoubleBufferedLayerStream
        from llama3fhe.application.session import _create_context, _encrypt_hidden
        from llama3fhe.application.settings import layer_schedule, resolve_settings
        from llama3fhe.backend import set_stage_sync
        from llama3fhe.layouts import AttentionPairLayout, FeatureMajorPrefillLayout
        from llama3fhe.model import Llama3Model, prepare_bootstrap_operator

        set_stage_sync(False)   # the operators' stage-timer device synchronisations (profiling only) off
        t0 = time.perf_counter()
        ref_args = resolve_poly_paths(build_parser(layer0_preset=True).parse_args(
            ["--key-mode", "host", "--seed", str(seed)]))
        self.feature, self.attention = FeatureMajorPrefillLayout(), AttentionPairLayout()
        self.config = Llama3CKKSConfig.from_json(ref_args.config)
        settings = resolve_settings(ref_args, self.config)
        self.schedule = layer_schedule(ref_args, settings)
        self.approx = ApproximationConfig(rmsnorm_path=ref_args.rms_coeffs, silu_path=ref_args.silu_coeffs,
                                          softmax_path=ref_args.softmax_coeffs)
        self.model = Llama3Model(config=self.config, num_layers=1, feature_layout=self.feature,
                                 attention_layout=self.attention)
        self.hidden, self.weights = _synthetic_inputs(int(ref_args.seed), layout=self.feature,
                                                      attention_layout=self.attention)
        self.rope_theta = float(getattr(ref_args, "rope_theta", 500000.0) or 500000.0)
        rotations = self.model.required_rotations(
            self.schedule, bootstrap_deep_level_budget=(3, 3) if self.schedule.softmax_main_deep_bootstrap else None)
        self.context = _create_context(self.config, rotations, auto_load_keys=settings.auto_load_keys)
        self.inputs = _encrypt_hidden(self.hidden, context=self.context, layout=self.feature,
                                      input_level=settings.input_level)
        self.bootstrap = prepare_bootstrap_operator(self.context, self.schedule)
        self.mask = _np.ones(int(self.feature.seq_len), dtype=bool)
        self._stream_cls = DoubleBufferedLayerStream
        self.rotation_keys = len(rotations)
        self.setup_seconds = time.perf_counter() - t0

    def release_transients(self) -> None:
        """Between steps: dead temporaries back to the allocator (the reference runner's
        ``_release_transient_device_memory``, ``llama3fhe/application/session.py``, without its ``empty_cache``:
        with expandable segments the pool does not fragment across steps, and handing the segments back to the driver
        makes the next step map them again, 0.6 s per layer), and the engine's reusable ModUp digits dropped, so that
        a step never reuses work of an earlier one (the same input ciphertexts are fed to every step)."""
        import gc

        import torch

        gc.collect()
        torch.cuda.synchronize()
        self.context.context.forget_digits()

    num_layers = 1

    def set_layers(self, n: int) -> None:
        """A model of ``n`` decoder layers (the same synthetic layer weights in every layer, layers after the first
        refreshing their input as the reference's model does)."""
        from llama3fhe.model import Llama3Model

        self.num_layers = int(n)
        self.model = Llama3Model(config=self.config, num_layers=self.num_layers, feature_layout=self.feature,
                                 attention_layout=self.attention)

    def layers(self):
        return self._stream_cls(loader=None, synthetic_weights=self.weights, approx_config=self.approx,
                                config=self.config, feature_layout=self.feature, attention_layout=self.attention,
                                num_layers=self.num_layers, rope_theta=self.rope_theta)

    def forward(self, inputs=None):
        return self.model.forward(self.hidden, crypto_context=self.context,
                                  input_ciphers=self.inputs if inputs is None else inputs, layers=self.layers(),
                                  bootstrap_operator=self.bootstrap, schedule=self.schedule, refresh_first_layer=False,
                                  attention_token_valid_mask=self.mask)

    def check(self, result) -> dict:
        """Decrypted layer output against the reference's own plaintext model of the same layer (its polynomial
        approximations, Alg2 softmax; ``llama3fhe/approx/layer.py:592-767``)."""
        from llama3fhe.application.client import decrypt_hidden
        from llama3fhe.approx.layer import poly_prefill_layer_numpy

        fhe = decrypt_hidden(result.ciphers, crypto_context=self.context, layout=self.feature)
        layer = next(iter(self.layers()))
        want = poly_prefill_layer_numpy(self.hidden, weights=layer.weights, approximations=layer.approximations,
                                        attention_layout=self.attention, layer_idx=0, rope_theta=self.rope_theta,
                                        use_alg2_softmax=True, token_valid_mask=self.mask).hidden
        err = np.abs(np.asarray(fhe, dtype=np.float64) - np.asarray(want, dtype=np.float64))
        scale = float(np.max(np.abs(want)))
        return {"max_abs_err": float(err.max()), "mean_abs_err": float(err.mean()), "max_abs_ref": scale,
                "max_rel_err": float(err.max() / scale) if scale else None}


def layer_cpu_rates(rows: int = 16, hoisted: int = 2, rotations: int = 1) -> dict:
    """CPU seconds per algorithmic byte of each kernel family, from the CPU restatement (oracle/, OpenMP, all host
    cores) on a bounded sample at the production chain's 13-limb linear level: the bytes of a sampled operation are
    counted with the same formulas the engine's per-family timers use (holmes_b200.fhe.OPTIMER)."""
    cpu = cpu_baseline(rows=rows, hoisted=hoisted, rotations=rotations)
    po = cpu["per_op_s"]
    N, cur, K, beta, slots = 1 << LOG_N, CUR_LIMBS, 8, 2, 1 << (LOG_N - 1)
    ks_bytes = (1 * (beta * (cur + K) + 2 * cur) + 2 * beta * (cur + K) + cur) * N * 8
    modup_bytes = (cur + beta * (cur + K)) * N * 8
    enc_bytes = 2 * slots * 16 + slots * 16 + cur * N * 8
    mac_bytes = (1 + 2 + 2) * cur * N * 8
    rates = {"keyswitch": po["hoisted_ks"] / ks_bytes, "modup": po["modup"] / modup_bytes,
             "encode_ntt": po["encode_row"] / enc_bytes, "fft_special": po["encode_row"] / enc_bytes,
             "bsgs_mac": po["mac_row_input"] / mac_bytes}
    rates["rescale"] = rates["keyswitch"]
    return {"rates_s_per_byte": rates, "cores": cpu["cores"], "per_op_s": po,
            "sample": f"{rows} rows encoded + MAC'd, 1 ModUp, {hoisted} hoisted + {rotations} full key switches at "
                      f"N=2^16 / 13 of 38 limbs"}


def layer_cpu_estimate(volume: dict, rates: dict) -> float:
    """Seconds of the CPU restatement for one layer: every family's algorithmic bytes in the layer times that
    family's CPU seconds per byte (families without a sampled rate use the key switch's)."""
    r = rates["rates_s_per_byte"]
    return float(sum(v["bytes"] * r.get(name, r["keyswitch"]) for name, v in volume.items()))


LAYER_VOLUME = os.path.join(ROOT, "profiles", "layer_op_volume.json")


def layer_cpu_rates_threads(threads: int, rows: int = 4):
    """``layer_cpu_rates`` measured in a child process limited to ``threads`` OpenMP threads (the thread count is
    fixed when the oracle's library first runs, so the parent's all-core library cannot be reused), or None."""
    env = dict(os.environ, OMP_NUM_THREADS=str(int(threads)), CUDA_VISIBLE_DEVICES="")
    try:
        res = subprocess.run([sys.executable, os.path.abspath(__file__), "--cpu-rates-json", "--cpu-rows", str(rows)],
                             env=env, capture_output=True, text=True, timeout=600)
        return json.loads(res.stdout.strip().splitlines()[-1]) if res.returncode == 0 else None
    except (subprocess.TimeoutExpired, ValueError, IndexError):
        return None


def write_kernel_list(setup, path: str) -> None:
    """One more (untimed) layer under CUPTI (torch.profiler, CUDA activity only): every kernel and copy with its
    launches, total device time and share, written to ``path`` as a markdown table.  The layer's ~360,000 launches
    make a per-launch ncu list impractical (its CSV alone runs to hundreds of MB); these are the same per-launch
    device durations, aggregated by kernel name."""
    import collections

    import torch
    from torch.profiler import ProfilerActivity, profile

    setup.release_transients()
    wall = time.perf_counter()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        setup.forward()
        torch.cuda.synchronize()
    wall = time.perf_counter() - wall
    agg = collections.defaultdict(lambda: [0, 0.0])
    first, last = None, None
    for e in prof.events():
        if e.device_type != torch.autograd.DeviceType.CUDA:
            continue
        rec = agg[e.name]
        rec[0] += 1
        rec[1] += float(getattr(e, "device_time_total", 0.0) or e.cuda_time_total)
        first = e.time_range.start if first is None else min(first, e.time_range.start)
        last = e.time_range.end if last is None else max(last, e.time_range.end)
    total = sum(v[1] for v in agg.values())
    lines = [f"device work {total / 1e6:.3f} s in a {((last or 0) - (first or 0)) / 1e6:.3f} s span "
             f"({sum(v[0] for v in agg.values())} launches and copies; wall {wall:.2f} s under the profiler)", "",
             "| kernel | launches | total ms | share |", "|---|---:|---:|---:|"]
    for name, (n, us) in sorted(agg.items(), key=lambda kv: -kv[1][1]):
        short = name if len(name) <= 110 else name[:107] + "..."
        lines.append(f"| `{short}` | {n} | {us / 1e3:.1f} | {us / total:.3f} |")
    with open(path, "w", encoding="utf-8") as f:
        f.write("\n".join(lines) + "\n")


def run_prefill_model(args) -> None:
    """BASELINE config 4 at world size 1, as a supplementary measurement: ``--layers`` decoder layers of the reference's
    own model (``Llama3Model.forward``, the synthetic one-layer preset's weights in every layer) on one GPU, after
    ``--warmup`` single-layer forwards (the keys of every layer are generated on first use there); ``--steps`` timed
    forwards of the whole model, CUDA events on the launching stream.  The full model takes minutes per step, so this
    is not the bench's default step."""
    import torch

    from holmes_b200 import _lib

    setup = _LayerSetup(seed=int(args.seed))
    for _ in range(max(1, args.warmup)):
        setup.forward()
    torch.cuda.synchronize()
    setup.set_layers(int(args.layers))
    clocks = ClockSampler(0)
    clocks.start()
    clocks.ready()
    n0 = ctypes_launches(_lib)
    times = []
    for _ in range(max(1, args.steps)):
        setup.release_transients()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        result = setup.forward()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) / 1e3)
        del result
    launches = (ctypes_launches(_lib) - n0) // max(1, args.steps)
    ck = clocks.stop()
    v = statistics.median(times)
    print(json.dumps({"metric": f"encrypted Llama-3-8B prefill-128 latency ({setup.num_layers} layers, 1 B200)",
                      "value": round(v, 3), "unit": "s", "n_gpus": 1, "steps": len(times),
                      "warmup": f"{max(1, args.warmup)} single-layer forward(s)", "higher_is_better": False,
                      "per_layer_s": round(v / setup.num_layers, 3), "step_times_s": [round(t, 3) for t in times],
                      "dtype": "u64 (RNS residues, 59/60-bit primes)",
                      "data": "synthetic (the reference's seeded one-layer preset's weights in every layer)",
                      "config": {"workload": f"BASELINE config 4 at world size 1: {setup.num_layers}-layer encrypted "
                                             "prefill of 128 tokens through the reference's Llama3Model.forward",
                                 "ckks": "N=2^16, 38 limbs, dnum 5, 59/60-bit"},
                      "gpu_launches": int(launches), "clocks": ck}), flush=True)


def run_layer(args) -> None:
    """BASELINE config 3 (see _LayerSetup): ``value`` = device seconds of one encrypted decoder layer with the 16
    input ciphertexts resident in HBM (CUDA events around each step on the launching stream, synchronised on both
    sides); ``e2e`` = the same through the public call with the input ciphertexts copied from pinned host memory and
    the output ciphertexts copied back inside every timed step.  The working set (keys, encoded weight chunks of
    GB each) is far above the 126 MB L2.  After the timed steps, one more step runs with the engine's per-family
    CUDA-event timers on (untimed) for the kernel breakdown and the roofline line.

    With N > 1 GPUs (torchrun) every rank runs its own replica of the layer on its own GPU: the reference's one-layer
    graph is a single-process program (its multi-GPU layer is the station chain of bench/t2_layer.py), so the N-GPU
    line reports the slowest replica's latency with per-GPU work fixed ("scaling": "weak", replicas only)."""
    import torch
    import torch.distributed as dist

    from holmes_b200 import _lib
    from holmes_b200 import fhe as F

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=900), device_id=torch.device("cuda", local))
    setup = _LayerSetup(seed=int(args.seed) + rank)
    steps, warm = max(1, args.steps), max(0, args.warmup)
    F.OPTIMER.enabled = False
    for _ in range(warm):
        setup.forward()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    def slowest(seconds: float) -> float:
        if world == 1:
            return seconds
        t = torch.tensor([seconds], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    clocks = ClockSampler(local)
    clocks.start()
    clocks.ready()
    barrier()
    n0 = ctypes_launches(_lib)
    mem0 = torch.cuda.memory_stats()
    times, result = [], None
    for _ in range(steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        result = None
        setup.release_transients()      # outside the timed interval, as the reference's runner does between samples
        a.record()
        result = setup.forward()
        b.record()
        torch.cuda.synchronize()
        times.append(slowest(a.elapsed_time(b) / 1e3))
    launches = (ctypes_launches(_lib) - n0) // steps
    mem1 = torch.cuda.memory_stats()
    memory = {"peak_allocated_gb": round(mem1.get("allocated_bytes.all.peak", 0) / 1e9, 1),
              "peak_reserved_gb": round(mem1.get("reserved_bytes.all.peak", 0) / 1e9, 1),
              **{k: (mem1.get(k, 0) - mem0.get(k, 0)) // steps
                 for k in ("num_alloc_retries", "num_device_alloc", "num_device_free", "num_sync_all_streams")}}
    ck = clocks.stop()
    # end to end: input ciphertexts from pinned host memory, outputs back to pinned host memory, every step
    host_in = [[c.cv[k].cpu().pin_memory() for k in range(2)] for c in setup.inputs]
    dev_in = tuple(c.cipher_like([torch.empty_like(c.cv[0]), torch.empty_like(c.cv[1])]) for c in setup.inputs)
    h2d = sum(int(t.numel()) * 8 for pair in host_in for t in pair)
    e2e_steps = max(1, min(steps, args.e2e_steps))
    e2e_times, d2h = [], 0
    barrier()
    for _ in range(e2e_steps):
        setup.release_transients()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for src, dst in zip(host_in, dev_in):
            dst.cv[0].copy_(src[0], non_blocking=True)
            dst.cv[1].copy_(src[1], non_blocking=True)
        out = setup.forward(dev_in)
        outs = [c.cv[k][:, :int(c.state.cur_limbs)].to("cpu", non_blocking=False) for c in out.ciphers
                for k in range(2)]
        b.record()
        torch.cuda.synchronize()
        d2h = sum(int(t.numel()) * 8 for t in outs)
        e2e_times.append(slowest(a.elapsed_time(b) / 1e3))
    # kernel-family breakdown: one more (untimed) step with the per-family CUDA-event timers
    # the same step also carries the reference's own stage timers, with their device synchronisations on
    from llama3fhe.backend import set_stage_sync

    F.OPTIMER.reset()
    F.OPTIMER.enabled = True
    setup.release_transients()
    set_stage_sync(True)
    prof = setup.forward()
    set_stage_sync(False)
    F.OPTIMER.enabled = False
    ops = F.OPTIMER.summary()
    phases = None
    try:
        phases = {str(k): round(float(v), 3) for k, v in prof.per_layer[0]["stage_seconds"].items()}
    except (AttributeError, IndexError, KeyError, TypeError, ValueError):
        pass
    del prof
    if args.kernel_list and rank == 0:
        write_kernel_list(setup, args.kernel_list)
    check = setup.check(result) if args.check and rank == 0 else None
    barrier()
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    v = statistics.median(times)
    hbm, kind = peaks()
    dominant = max(ops.items(), key=lambda kv: kv[1]["ms"]) if ops else None
    roofline = None
    if dominant:
        name, d = dominant
        per_launch_s = d["ms"] / 1e3 / d["launches"]
        achieved = d["bytes"] / d["launches"] / per_launch_s / 1e9
        roofline = {"bound": "hbm", "kernel": name, "achieved": round(achieved, 1), "peak": hbm, "peak_kind": kind,
                    "unit": "GB/s", "frac": round(achieved / hbm, 4),
                    "traffic": measured_traffic(name, d["bytes"] // d["launches"]),
                    "algorithmic_bytes_per_launch": d["bytes"] // d["launches"],
                    "avg_launch_ms": round(d["ms"] / d["launches"], 4),
                    "share_of_step": round(d["ms"] / 1e3 / v, 4)}
    volume = {k: {"launches": val["launches"], "bytes": val["bytes"], "ms": round(val["ms"], 2)}
              for k, val in ops.items()}
    cpu = None
    if args.cpu_baseline and world == 1:
        rates = layer_cpu_rates()
        cpu = {"value": round(layer_cpu_estimate(volume, rates), 1), "unit": "s", "cores": rates["cores"],
               "kind": "port",
               "sample": rates["sample"] + "; scaled to the layer by every kernel family's algorithmic bytes in one "
                                           "layer (CPU seconds per byte of that family times its bytes)",
               "per_op_s": rates["per_op_s"]}
        one = layer_cpu_rates_threads(1, rows=16)
        if one is not None:
            cpu["one_thread"] = {"value": round(layer_cpu_estimate(volume, one), 1), "unit": "s", "cores": 1,
                                 "sample": one["sample"], "per_op_s": one["per_op_s"]}
    line = {"metric": LAYER_METRIC, "value": round(v, 4), "unit": "s", "n_gpus": world, "steps": steps,
            "warmup": warm, "ms_per_step": round(v * 1e3, 1), "higher_is_better": False,
            "scaling": "weak" if world > 1 else "strong", "vs_baseline": None,
            "dtype": "u64 (RNS residues, 59/60-bit primes)",
            "data": "synthetic (the reference's seeded one-layer preset: weights ~N(0, 0.002^2), hidden ~N(0, 0.01^2))",
            "config": {"workload": "BASELINE config 3: one Llama-3-8B decoder layer, encrypted prefill of 128 tokens, "
                                   "1 B200 -- the reference's own layer graph (llama3fhe TransformerLayer.forward / "
                                   "graph.prefill.evaluate, run_layer0 synthetic preset) on libholmes_cuda",
                       "geometry": "hidden 4096, 32 q / 8 kv heads x 128, MLP 14336, 128 tokens in 16 FM ciphertexts",
                       "ckks": f"N=2^16, {setup.context.context.L} limbs, dnum 5, 59/60-bit",
                       "parallelism": f"replicas x{world} (one independent layer per GPU)" if world > 1 else "1 GPU",
                       "rotation_keys": setup.rotation_keys, "keys": "generated on first use, trimmed to their level",
                       "l2": "working set (keys, encoded weight chunks, bootstrap constants) >> 126 MB L2"},
            "roofline": roofline,
            "kernels": {k: {"launches": val["launches"], "ms_per_step": round(val["ms"], 2)} for k, val in ops.items()},
            "cpu_baseline": cpu, "gpu_launches": int(launches), "clocks": ck,
            "e2e": {"value": round(statistics.median(e2e_times), 4), "unit": "s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps, "step_times_s": [round(t, 3) for t in e2e_times]},
            "setup_s": round(setup.setup_seconds, 1), "step_times_s": [round(t, 3) for t in times],
            "device_memory_per_step": memory,
            "phases_s": phases}
    if check is not None:
        line["parity_vs_reference_poly_model"] = check
    if args.write_volume:
        with open(LAYER_VOLUME, "w", encoding="utf-8") as f:
            json.dump({"what": "per kernel family of one config-3 layer on the engine: launches, algorithmic bytes "
                               "and device ms (holmes_b200.fhe.OPTIMER)", "families": volume}, f, indent=1)
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_reference_layer(args) -> None:
    """The reference arm for the layer workload: EasyFHE (the reference's engine) is not distributed, so the CPU
    restatement stands in -- sampled per-family CPU rates (all host cores) times the per-family algorithmic bytes of
    one layer (profiles/layer_op_volume.json, recorded from the engine's run of the same layer)."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    with open(LAYER_VOLUME, encoding="utf-8") as f:
        volume = json.load(f)["families"]
    for _ in range(min(1, args.warmup)):
        layer_cpu_rates(rows=2, hoisted=1, rotations=1)
    vals, rates = [], None
    for _ in range(max(1, min(args.steps, 3))):
        rates = layer_cpu_rates()
        vals.append(layer_cpu_estimate(volume, rates))
    v = round(statistics.median(vals), 1)
    line = {"impl": "reference", "metric": LAYER_METRIC, "value": v, "unit": "s",
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "u64 (RNS residues)",
            "data": "synthetic (seeded)",
            "config": {"workload": "BASELINE config 3 layer, estimated on the CPU restatement of the reference's "
                                   "engine (EasyFHE is not distributed and cannot run here)"},
            "cpu_baseline": {"value": v, "unit": "s", "cores": rates["cores"], "kind": "port",
                             "sample": rates["sample"] + "; scaled by the layer's per-family algorithmic bytes "
                                                         "(profiles/layer_op_volume.json)"},
            "e2e": {"value": v, "unit": "s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def ctypes_launches(lib) -> int:
    import ctypes as _ct

    n = _ct.c_ulonglong()
    lib.call("holmes_launch_count", _ct.byref(n))
    return int(n.value)


def run_primitives(args) -> None:
    """BASELINE config 2, the RNS-CKKS primitive sweep: N = 2^16, ~50-bit primes, dnum 3 (alpha = K = 12),
    L = 1..36 active limbs, residues uniform in [0, q_i) (seed 0).  Per L: batched forward / inverse NTT,
    a rotation (hoisted-free key switch) of a batch of 16 ciphertexts sharing one key, the plaintext x
    ciphertext product and a rescale, each timed with CUDA events after a warm-up (inputs above L2 at the
    larger sizes).  Algorithmic bytes per op: NTT 16 b L N; key switch per ciphertext
    (L + 2 beta (L + K) / batch + L + 2 L) N 8 with the key read once per batch; plaintext product 5 L N 8;
    rescale (2 L + 2 (L - 1)) N 8.  One JSON line with a row per (op, L)."""
    import torch

    from holmes_b200 import _lib as L_
    from holmes_b200 import fhe as F

    peak, peak_kind = peaks()
    lmax = 36
    spec = F.CKKSContextSpec(depth=lmax - 1, log_n=16, dnum=3, dcrt_bits=50, first_mod=50, special_bits=50, seed=0,
                             hamming_weight=192, auto_load_keys=False)
    client, ctx = F.generate_client_context(spec)
    N, K = ctx.N, ctx.K
    gen = torch.Generator(device=ctx.device).manual_seed(0)
    qcol = torch.tensor(list(ctx.moduli[:lmax]), dtype=torch.int64, device=ctx.device).view(1, lmax, 1)

    def rand(items, limbs):
        r = torch.randint(0, 2 ** 62, (items, limbs, N), device=ctx.device, dtype=torch.int64, generator=gen)
        return (r % qcol[:, :limbs]).to(torch.uint64)

    def timed(fn, reps):
        fn()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / reps / 1e3

    rows = []

    def row(op, limbs, batch, seconds, nbytes, units):
        rows.append({"op": op, "limbs": limbs, "batch": batch, "ms": round(seconds * 1e3, 4),
                     "ops_per_s": round(units / seconds, 1), "gbs": round(nbytes / seconds / 1e9, 1),
                     "hbm_frac": round(nbytes / seconds / 1e9 / peak, 4)})

    for limbs in (1, 4, 8, 16, 24, 36):
        for b in (1, 16, 256 if limbs <= 8 else 64):
            x = rand(b, limbs)
            for inv in (0, 1):
                t = timed(lambda: L_.call("holmes_ntt", ctx.handle, x.data_ptr(), b, limbs, limbs * N, 0, inv, 0), 5)
                row("intt" if inv else "ntt", limbs, b, t, 16 * b * limbs * N, b * limbs)
            del x
        I = 16
        c0, c1 = rand(I, limbs), rand(I, limbs)
        o0, o1 = torch.empty_like(c0), torch.empty_like(c1)
        g = ctx.galois(1)
        key = ctx.switch_key(g, limbs)
        beta = ctx.beta(limbs)
        t = timed(lambda: F.rotate_batch(ctx, c0, c1, limbs, 1, o0, o1), 3)
        row("rotate", limbs, I, t, (I * 4 * limbs + 2 * beta * (limbs + K)) * N * 8, I)
        ct = F.Cipher([c0, c1], F.CipherState(limbs, 1, ctx.scale), ctx.max_slots, False, I, ctx)
        pt = F.Plaintext([rand(1, limbs)], F.CipherState(limbs, 1, ctx.scale), ctx.max_slots, False, 1, ctx)
        t = timed(lambda: F.homo_mul_pt(ct, pt, ctx), 5)
        row("mul_pt", limbs, I, t, (limbs + 4 * limbs * I) * N * 8, I)
        if limbs >= 2:
            ct2 = F.Cipher([c0, c1], F.CipherState(limbs, 2, ctx.scale ** 2), ctx.max_slots, False, I, ctx)
            t = timed(lambda: F.rescale(ct2, ctx), 5)
            row("rescale", limbs, I, t, I * (4 * limbs - 2) * N * 8, I)
        del c0, c1, o0, o1, key
    print(json.dumps({"workload": "primitives (config 2)", "n": N, "dnum": 3, "alpha": ctx.alpha, "K": K,
                      "peak_gbs": peak, "peak_kind": peak_kind, "rows": rows}), flush=True)
    ctx.close()


def run_bootstrap(args) -> None:
    """Production-size bootstrap: N = 2^16, 38 limbs (59/60-bit, dnum 5), level budget (5, 5) -> 18 limbs left
    (llama3fhe/parallel/presets.py:25-60), a batch of ``--boot-batch`` ciphertexts refreshed together
    (BootstrapOperator.refresh_many, the pair-refresh call of parallel/prefill/stations.py:102-174)."""
    import torch

    from holmes_b200 import bootstrap as BS
    from holmes_b200 import fhe as F
    from holmes_b200 import linear as LN

    spec = F.CKKSContextSpec(depth=DEPTH, log_n=LOG_N, dnum=DNUM, dcrt_bits=DCRT, first_mod=FIRST, special_bits=60,
                             hamming_weight=192, seed=0, auto_load_keys=False)
    client, ctx = F.generate_client_context(spec)
    session = LN.Session(client, ctx)
    t0 = time.perf_counter()
    op = BS.BootstrapOperator.prepare(session, BS.BootstrapConfig(log_slots=15, level_budget=(5, 5)))
    torch.cuda.synchronize()
    setup = time.perf_counter() - t0
    rng = np.random.default_rng(0)
    zs = [(rng.normal(size=ctx.max_slots) + 1j * rng.normal(size=ctx.max_slots)) * 0.5 for _ in range(args.boot_batch)]
    cts = [client.encrypt(z, cur_limbs=3, counter=i) for i, z in enumerate(zs)]
    it = int(args.boot_iterations)
    for _ in range(max(1, args.warmup)):
        op.refresh_many(cts, iterations=it)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(args.steps):
        outs = op.refresh_many(cts, iterations=it)
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / args.steps
    err = max(float(np.abs(client.decrypt(o) - z).max()) for o, z in zip(outs, zs))
    print(json.dumps({"metric": "CKKS bootstrap latency per ciphertext (full slots, N=2^16, 38 -> 18 limbs)",
                      "value": round(ms / 1e3 / len(cts), 5), "unit": "s", "batch": len(cts),
                      "ms_per_batch": round(ms, 2), "steps": args.steps, "higher_is_better": False,
                      "max_abs_err": err, "setup_s": round(setup, 1), "rotation_keys": len(op.program.rotations),
                      "key_gb": round(ctx.key_bytes / 1e9, 1), "depth": op.program.spec.depth,
                      "iterations": it, "output_limbs": int(outs[0].state.cur_limbs)}), flush=True)
    ctx.close()


def run_silu(args) -> None:
    """SiLU of the model's MLP as the reference evaluates it (operators/nonlinear/polynomial.py:469-562): a degree-236
    Chebyshev series on [-8, 8] (k = 16, m = 4: 8 levels + 1 for the map) over ``--inputs`` ciphertexts at once,
    N = 2^16, entering at 18 limbs (a refresh's output level) of the production 38-limb chain.  Decoded against the
    float64 series."""
    import torch
    from numpy.polynomial import chebyshev as npcheb

    from holmes_b200 import _lib
    from holmes_b200 import fhe as F
    from holmes_b200 import polynomial as P

    spec = F.CKKSContextSpec(depth=DEPTH, log_n=LOG_N, dnum=DNUM, dcrt_bits=DCRT, first_mod=FIRST, special_bits=60,
                             hamming_weight=192, seed=0, auto_load_keys=False)
    client, ctx = F.generate_client_context(spec)
    a, b, degree, limbs = -8.0, 8.0, 236, 18
    std = npcheb.chebinterpolate(lambda y: (v := (y * (b - a) + (a + b)) / 2) / (1 + np.exp(-v)), degree)
    ref = std.copy()
    ref[0] *= 2.0
    rng = np.random.default_rng(0)
    xs = [rng.uniform(a, b, size=ctx.max_slots) for _ in range(args.inputs)]
    batch = F.pack_cipher_batch([client.encrypt(x, cur_limbs=limbs, counter=i) for i, x in enumerate(xs)])
    for _ in range(max(1, args.warmup)):
        P.eval_chebyshev_series_cipher(batch, ref, lower_bound=a, upper_bound=b, crypto_context=ctx)
    torch.cuda.synchronize()
    count0 = _lib.ctypes.c_ulonglong()
    _lib.call("holmes_launch_count", _lib.ctypes.byref(count0))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        out = P.eval_chebyshev_series_cipher(batch, ref, lower_bound=a, upper_bound=b, crypto_context=ctx)
    e1.record()
    torch.cuda.synchronize()
    count1 = _lib.ctypes.c_ulonglong()
    _lib.call("holmes_launch_count", _lib.ctypes.byref(count1))
    ms = e0.elapsed_time(e1) / args.steps
    err = max(float(np.abs(client.decrypt(out, item=i).real - npcheb.chebval((2 * x - a - b) / (b - a), std)).max())
              for i, x in enumerate(xs[:2]))
    print(json.dumps({"metric": "SiLU (degree-236 Chebyshev, Paterson-Stockmeyer) latency per ciphertext, N=2^16",
                      "value": round(ms / 1e3 / args.inputs, 6), "unit": "s", "batch": args.inputs,
                      "ms_per_batch": round(ms, 2), "steps": args.steps, "higher_is_better": False,
                      "input_limbs": limbs, "output_limbs": int(out.state.cur_limbs), "max_abs_err_vs_series": err,
                      "gpu_launches": int((count1.value - count0.value) // max(1, args.steps))}), flush=True)
    ctx.close()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", choices=("linear", "layer", "bootstrap", "primitives", "silu"), default=None,
                    help="default: layer (BASELINE config 3) when the reference's application is installed in "
                         "baseline/_ref, else linear (one QKV page)")
    ap.add_argument("--boot-batch", type=int, default=8)
    ap.add_argument("--boot-iterations", type=int, default=1, help="2 = Meta-BTS correction")
    ap.add_argument("--kernel", default=None, help="profile one kernel family (see run_kernel)")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("holmes", "reference"), default="holmes")
    ap.add_argument("--inputs", type=int, default=INPUTS)
    ap.add_argument("--limbs", type=int, default=CUR_LIMBS)
    ap.add_argument("--parallelism", choices=("token", "chunk"), default="chunk")
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--cpu-rows", type=int, default=128, help="diagonal rows in the CPU baseline's sample")
    ap.add_argument("--no-check", dest="check", action="store_false")
    ap.add_argument("--seed", type=int, default=26081461, help="seed of the layer workload's synthetic preset")
    ap.add_argument("--e2e-steps", type=int, default=3, help="end-to-end steps of the layer workload")
    ap.add_argument("--write-volume", action="store_true",
                    help="layer workload: record the per-family volume of one layer in profiles/layer_op_volume.json")
    ap.add_argument("--vs-ref", action="store_true",
                    help="with --kernel mac|encode: time the reference's in-tree kernel beside the engine's")
    ap.add_argument("--layers", type=int, default=1,
                    help="layer workload: decoder layers per step (> 1: the supplementary config-4 run at world size 1)")
    ap.add_argument("--kernel-list", default=None,
                    help="layer workload: write the per-kernel device time of one more (untimed) layer to this file")
    ap.add_argument("--cpu-rates-json", action="store_true", help=argparse.SUPPRESS)
    args = ap.parse_args()
    if args.cpu_rates_json:    # one bounded CPU sample in this process's thread count (OMP_NUM_THREADS)
        print(json.dumps(layer_cpu_rates(rows=args.cpu_rows)), flush=True)
        return
    if args.workload is None:
        args.workload = "layer" if os.path.isdir(os.path.join(ROOT, "baseline", "_ref", "llama3fhe")) else "linear"
    if args.workload == "layer":
        # the layer's many short-lived multi-GB temporaries fragment a fixed-segment pool
        os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    if args.kernel and args.vs_ref:
        run_vs_ref(args)
    elif args.kernel:
        run_kernel(args)
    elif args.workload == "layer" and args.layers > 1 and args.impl != "reference":
        run_prefill_model(args)
    elif args.workload == "layer":
        run_reference_layer(args) if args.impl == "reference" else run_layer(args)
    elif args.workload == "bootstrap":
        run_bootstrap(args)
    elif args.workload == "primitives":
        run_primitives(args)
    elif args.workload == "silu":
        run_silu(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_engine(args)


if __name__ == "__main__":
    main()
