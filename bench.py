#!/usr/bin/env python3
"""Sparse-FFN layer benchmark (BASELINE metric: tokens/s per layer and the
fraction of the HBM roofline on active-weight bytes).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--model 7b] [--batch B] [--activity 0.10] [--path auto]
                    [--wtype f16|q8_0|q4_0] [--predictor] [--shard] [--config 1..5]

--config N applies BASELINE.json configuration N (1: 7B B=1 with the
predictor, 2: 7B B=32 -- the default --, 3: 13B B=64 8% with a predictor per
layer over 40 layers, 4: 7B Q4_0, 5: 70B neuron-sharded); explicit flags win.

A step is one sparse FFN layer (union -> gathered gate/up -> ReLU*up ->
gathered down) over one batch of B tokens.  Steps rotate over L distinct
layer copies (own weights, own Zipf(0.8) activity) so the weights read per
cycle exceed the 126 MB L2 several times: no step reads another step's
weights from L2.  Timing: CUDA events on the launching stream around exactly
K steps replayed from CUDA graphs, barrier + synchronize on both sides, max
over ranks.  Under torchrun each rank runs its own replica of the workload
(the config-2 layer does not shard): scaling "weak".

--impl reference times the reference's CPU path (a PyTorch masked-dense FFN
on all host cores; the reference itself has no CPU FFN and its GPU code is
not a CPU path) on the same config; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "sparse-FFN tokens/s per layer vs batch; % HBM roofline on active bytes"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=40000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", default="7b")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--activity", type=float, default=0.10)
    ap.add_argument("--path", choices=["auto", "gemv", "tensor"], default="auto")
    ap.add_argument("--per-token", type=int, default=1)
    ap.add_argument("--layers", type=int, default=0, help="distinct layer copies rotated (0 = auto)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--shard", action="store_true",
                    help="shard the layer's neurons across the torchrun ranks (config 5) instead of replicas")
    ap.add_argument("--wtype", choices=["f16", "q8_0", "q4_0"], default="f16",
                    help="weight format (config 4: ggml block quantisation of fp32 N(0, 0.02^2) weights)")
    ap.add_argument("--predictor", action="store_true",
                    help="run the DejaVu predictor (P1 [1024][d], P2 [f][1024], top-k per token) ahead of each "
                         "layer; its labels feed the FFN and its bytes count in the roofline (configs 1 and 3)")
    ap.add_argument("--config", type=int, default=0, choices=[0, 1, 2, 3, 4, 5],
                    help="BASELINE.json configuration preset (0: the flags as given)")
    a = ap.parse_args()
    presets = {
        1: dict(model="7b", batch=1, activity=0.10, predictor=True),
        2: dict(model="7b", batch=32, activity=0.10),
        3: dict(model="13b", batch=64, activity=0.08, predictor=True, layers=40),
        4: dict(model="7b", batch=32, activity=0.10, wtype="q4_0"),
        5: dict(model="70b", batch=32, activity=0.10, shard=True),
    }
    given = {k.lstrip("-").replace("-", "_") for k in sys.argv[1:] if k.startswith("--")}
    for k, v in presets.get(a.config, {}).items():
        if k not in given:
            setattr(a, k, v)
    return a


PRED_RANK = 1024  # DejaVu predictor rank D (BASELINE configs 1 and 3)


def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def workload_name(a, U):
    wt = {"f16": "fp16 weights", "q8_0": "Q8_0 weights", "q4_0": "Q4_0 weights"}[a.wtype]
    act = (f"{a.activity:.0%} per-token activity from the DejaVu predictor (top-k, run ahead of the layer)"
           if a.predictor else f"{a.activity:.0%} per-token activity Zipf(0.8)")
    return f"{a.model} sparse FFN layer (ReLU-gated SwiGLU), B={a.batch}, {wt}, {act}, union U~{U}"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class Clocks:
    """Samples SM clocks and throttle reasons with nvidia-smi during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = os.path.join(ROOT, "gpurun_out", f"clocks_{os.getpid()}.csv")

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.fh.close()

    def summary(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                rows.append((float(f[1]), float(f[2]), f[5:9]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i in range(4) if r[i].lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "reasons": reasons, "samples": len(rows)}


def make_layers(a, L, device, rank, world=1):
    """L distinct layer copies.  Replicas: each rank its own layer.  Sharded:
    labels and x are the same on every rank (seeds without the rank) and the
    rank holds only its rows of the weights."""
    import torch
    from spbatch_b200.shard import shard_range
    from spbatch_b200.workload import SHAPES, zipf_active_labels
    d, f = SHAPES[a.model]["d"], SHAPES[a.model]["f"]
    k = int(round(a.activity * f))
    seed = 0 if a.shard else rank
    f0, f1 = shard_range(f, world, rank) if a.shard else (0, f)
    import spbatch_b200 as spb
    gen = torch.Generator(device=device)
    gen.manual_seed(1234 + rank)
    quant = None
    if a.wtype != "f16":
        # ggml block quantisation of one fp32 N(0, 0.02^2) set (host quantiser,
        # byte-identical to the oracle); every layer gets its own copy, so the
        # rotation still touches distinct addresses
        wt = spb.W_Q8_0 if a.wtype == "q8_0" else spb.W_Q4_0
        quant = [torch.from_numpy(spb.quantize((torch.randn((f1 - f0, d), generator=gen, device=device) * 0.02)
                                               .cpu().numpy(), wt)).to(device) for _ in range(3)]
    pws = spb.predict_workspace(a.batch, PRED_RANK, f1 - f0, device) if a.predictor else None
    layers = []
    for l in range(L):
        if quant is not None:
            W = [q.clone() for q in quant]
        else:
            W = [(torch.randn((f1 - f0, d), generator=gen, device=device) * 0.02).half() for _ in range(3)]
        x_np = np.random.default_rng([seed, l]).standard_normal((a.batch, d)).astype(np.float32)
        x = torch.from_numpy(x_np).to(device)
        P = None
        if a.predictor:
            # DejaVu low-rank predictor: P1 [D][d] ~ N(0, 1/d), P2 [f][D] ~ N(0, 1/D); its per-token
            # top-k labels drive this layer
            P = [(torch.randn((PRED_RANK, d), generator=gen, device=device) / math.sqrt(d)).half(),
                 (torch.randn((f1 - f0, PRED_RANK), generator=gen, device=device) / math.sqrt(PRED_RANK)).half()]
            lab = spb.predict(P[0], P[1], x, k=k, workspace=pws)
            torch.cuda.synchronize()
            lab_np = lab.cpu().numpy()
            lab_full = lab_np
        else:
            lab_full = zipf_active_labels(a.batch, f, k, seed=seed, layer=l)
            lab_np = np.ascontiguousarray(lab_full[:, f0:f1])
            lab = torch.from_numpy(lab_np).to(device)
        layers.append(dict(i=l, W=W, P=P, lab_np=lab_np, x_np=x_np, U=int((lab_np > 0).any(0).sum()),
                           U_full=int((lab_full > 0).any(0).sum()), lab=lab, x=x,
                           out=torch.empty((a.batch, d), device=device)))
    return d, f1 - f0, k, layers, pws


def run_ours(a):
    import torch
    import spbatch_b200 as spb
    from spbatch_b200.workload import active_bytes

    ws_n, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if ws_n > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=device)
    path = {"auto": spb.PATH_AUTO, "gemv": spb.PATH_GEMV, "tensor": spb.PATH_TENSOR}[a.path]

    from spbatch_b200.workload import SHAPES
    d0, f0 = SHAPES[a.model]["d"], SHAPES[a.model]["f"]
    wb = {"f16": 2.0, "q8_0": 34 / 32, "q4_0": 18 / 32}[a.wtype]
    est = active_bytes(d0, min(f0, int(a.activity * f0 * min(a.batch, 8))), a.batch, wb,
                       (d0 * PRED_RANK + PRED_RANK * f0) * 2 if a.predictor else 0)
    if a.shard:
        est /= ws_n
    L = a.layers or int(min(32, max(4, math.ceil(3 * L2_BYTES / est))))
    d, f, k, layers, pws = make_layers(a, L, device, rank, ws_n)
    wtype = {"f16": spb.W_F16, "q8_0": spb.W_Q8_0, "q4_0": spb.W_Q4_0}[a.wtype]
    w_bytes = {"f16": 2.0, "q8_0": 34 / 32, "q4_0": 18 / 32}[a.wtype]
    pred_bytes = (d * PRED_RANK + PRED_RANK * f) * 2 if a.predictor else 0
    ws = spb.new_workspace(a.batch, d, f, 0, device)
    Us = [ly["U"] for ly in layers]
    bytes_per_step = float(np.mean([active_bytes(d, U, a.batch, w_bytes, pred_bytes) for U in Us]))

    sharded = a.shard and ws_n > 1

    def fwd(ly, x=None, out=None):
        o = ly["out"] if out is None else out
        xx = ly["x"] if x is None else x
        if a.predictor:  # labels of this step from the layer's predictor
            spb.predict(ly["P"][0], ly["P"][1], xx, k=k, out=ly["lab"], workspace=pws)
        spb.ffn_forward(*ly["W"], xx, ly["lab"], wtype=wtype, out=o,
                        per_token_mask=bool(a.per_token), path=path, workspace=ws)
        if sharded:  # one all-reduce of the [B][d] partial outputs (NCCL)
            torch.distributed.all_reduce(o)

    stream = torch.cuda.Stream(device)
    with torch.cuda.stream(stream):
        for i in range(max(3, a.warmup)):
            fwd(layers[i % L])
    torch.cuda.synchronize()

    K = a.steps
    full, rem = divmod(K, L)

    def capture(n, body):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(n):
                body(layers[i % L])
        return g

    class Eager:
        """Stands in for a graph when steps contain a collective: they are
        launched eagerly instead of being captured."""

        def __init__(self, n, body):
            self.n, self.body = n, body

        def replay(self):
            for i in range(self.n):
                self.body(layers[i % L])

    if sharded:
        capture = Eager  # noqa: F811  (collectives stay out of graph capture)
    g_full = capture(L, fwd) if full else None
    g_rem = capture(rem, fwd) if rem else None

    def timed(gf, gr):
        if ws_n > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):  # graphs replay on the current stream
            e0.record(stream)
            for _ in range(full):
                gf.replay()
            if gr is not None:
                gr.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if ws_n > 1:
            t = torch.tensor([ms], device=device)
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            torch.distributed.barrier()
            ms = float(t.item())
        return ms

    # untimed replays, then the timed region with clocks sampled
    with torch.cuda.stream(stream):
        for gr in (g_full, g_rem):
            if gr is not None:
                gr.replay()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        ms = timed(g_full, g_rem)
    clocks = clk.summary()

    # e2e: host-pinned inputs copied in and the output copied back every step
    pinned = [dict(x=torch.from_numpy(ly["x_np"]).pin_memory(), lab=torch.from_numpy(ly["lab_np"]).pin_memory(),
                   out=torch.empty((a.batch, d)).pin_memory()) for ly in layers]
    xin = [torch.empty_like(ly["x"]) for ly in layers]
    labin = [torch.empty_like(ly["lab"]) for ly in layers]

    def e2e_body(ly):
        i = ly["i"]
        xin[i].copy_(pinned[i]["x"], non_blocking=True)
        if a.predictor:  # labels are produced on the device from x
            spb.predict(ly["P"][0], ly["P"][1], xin[i], k=k, out=labin[i], workspace=pws)
        else:
            labin[i].copy_(pinned[i]["lab"], non_blocking=True)
        spb.ffn_forward(*ly["W"], xin[i], labin[i], wtype=wtype, out=ly["out"], per_token_mask=bool(a.per_token),
                        path=path, workspace=ws)
        if sharded:
            torch.distributed.all_reduce(ly["out"])
        pinned[i]["out"].copy_(ly["out"], non_blocking=True)

    with torch.cuda.stream(stream):
        for ly in layers:
            e2e_body(ly)
    torch.cuda.synchronize()
    ge_full = capture(L, e2e_body) if full else None
    ge_rem = capture(rem, e2e_body) if rem else None
    ms_e2e = timed(ge_full, ge_rem)

    tokens = a.batch * K * (1 if sharded else ws_n)
    value = tokens / (ms / 1e3)
    peak, peak_kind = hbm_peak()
    t_step = ms / K / 1e3
    achieved = bytes_per_step / t_step / 1e9
    launches_per_step = spb.lib().spb_ffn_launches(a.batch, d, wtype, path)
    if a.predictor:
        launches_per_step += 3  # predictor: hidden layer, logits, top-k selection
    rec = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws_n, "steps": K, "warmup": a.warmup,
        "ms_per_step": ms / K, "higher_is_better": True, "scaling": "strong" if sharded else "weak",
        "vs_baseline": None, "dtype": a.wtype,
        "data": "synthetic (seeded N(0,0.02^2) fp16 weights, N(0,1) x, Zipf(0.8) activity; no dataset)",
        "config": {"workload": workload_name(a, int(np.mean([ly["U_full"] for ly in layers]))), "d": d,
                   "f_per_gpu": f, "batch": a.batch,
                   "k_per_token": k, "union_mean": float(np.mean(Us)), "layers_rotated": L,
                   "per_token_mask": bool(a.per_token), "path": a.path, "weights": a.wtype,
                   "predictor": (f"DejaVu rank {PRED_RANK}, top-{k} per token, run ahead of every layer "
                                 f"({pred_bytes / 1e6:.1f} MB per layer counted in bytes_per_step)"
                                 if a.predictor else None),
                   "l2": f"inputs larger than L2: {L} layer copies rotated, "
                         f"{L * bytes_per_step / 1e6:.0f} MB touched per cycle vs 126 MB L2",
                   "parallelism": (f"neuron-sharded tp{ws_n} + NCCL all-reduce" if sharded else
                                   f"replicas x{ws_n}" if ws_n > 1 else "single GPU")},
        "roofline": {"bound": "hbm", "kernel": "whole layer (union + gate/up + down launches)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} hbm_gbs", "traffic": traffic_from_profiles(a),
                     "bytes_per_step": bytes_per_step},
        "e2e": {"value": tokens / (ms_e2e / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": a.batch * d * 4 + (0 if a.predictor else a.batch * f * 4),
                "d2h_bytes_per_step": a.batch * d * 4,
                "ms_per_step": ms_e2e / K},
        "clocks": clocks,
        "gpu_launches": launches_per_step * K,
    }
    if rank == 0 and ws_n == 1 and not a.no_cpu:
        rec["cpu_baseline"] = cpu_baseline(a, layers[0], budget=a.cpu_budget)
    if rank == 0:
        print(json.dumps(rec), flush=True)
    if ws_n > 1:
        torch.distributed.destroy_process_group()


def traffic_from_profiles(a):
    """DRAM bytes per layer from the committed ncu summary, when one exists for this workload."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as fh:
            t = json.load(fh)
        return t.get(f"{a.model}_b{a.batch}_{a.path}")
    except Exception:
        return None


def cpu_baseline(a, ly, budget=15.0):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from cpu_ffn import MaskedDenseFFN, time_steps
    if a.wtype == "f16":
        W = [w.float().cpu().numpy() for w in ly["W"]]
    else:  # the CPU baseline computes with the dequantised weights (oracle dequantisation)
        import oracle
        qt = 8 if a.wtype == "q8_0" else 4
        d = ly["x_np"].shape[1]
        W = [oracle.dequantize(w.cpu().numpy(), qt, d) for w in ly["W"]]
    ffn = MaskedDenseFFN(*W)
    n, s = time_steps(ffn, ly["x_np"], ly["lab_np"], budget_s=budget)
    return {"value": a.batch * n / s, "unit": "tokens/s", "cores": ffn.threads, "kind": "port",
            "sample": f"{n} whole steps (one {a.model} layer, B={a.batch}) in {s:.1f} s, PyTorch fp32 "
                      f"masked-dense FFN on {ffn.threads} host threads"}


def run_reference(a):
    ws_n, rank, _ = dist_env()
    if rank != 0:
        return
    import torch
    from spbatch_b200.workload import SHAPES, zipf_active_labels
    d, f = SHAPES[a.model]["d"], SHAPES[a.model]["f"]
    k = int(round(a.activity * f))
    g = torch.Generator().manual_seed(1234)
    W = [(torch.randn((f, d), generator=g) * 0.02).half().float().numpy() for _ in range(3)]
    lab = zipf_active_labels(a.batch, f, k, seed=0, layer=0)
    x = np.random.default_rng([0, 0]).standard_normal((a.batch, d)).astype(np.float32)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from cpu_ffn import MaskedDenseFFN, time_steps
    ffn = MaskedDenseFFN(*W)
    for _ in range(min(a.warmup, 3)):
        ffn(x, lab)
    n, s = time_steps(ffn, x, lab, budget_s=min(120.0, max(10.0, a.cpu_budget * 4)), max_steps=a.steps)
    value = a.batch * n / s
    U = int((lab > 0).any(0).sum())
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws_n, "steps": n,
        "warmup": min(a.warmup, 3), "ms_per_step": s / n * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload_name(a, U), "d": d, "f": f, "batch": a.batch, "k_per_token": k},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": ffn.threads, "kind": "port",
                         "sample": f"{n} of the requested {a.steps} steps (time-bounded), PyTorch fp32 "
                                   f"masked-dense FFN restating MLP_naive on {ffn.threads} host threads"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    a = parse()
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
