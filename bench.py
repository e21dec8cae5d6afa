#!/usr/bin/env python3
"""Sparse-FFN layer benchmark (BASELINE metric: tokens/s per layer and the
fraction of the HBM roofline on active-weight bytes).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--model 7b] [--batch B] [--activity 0.10] [--path auto]
                    [--wtype f16|q8_0|q4_0] [--predictor] [--shard] [--replicas]
                    [--config 1..5] [--no-sweep] [--no-dense] [--no-cpu]

--config N applies BASELINE.json configuration N (1: 7B B=1 with the
predictor, 2: 7B B=32 -- the default --, 3: 13B B=64 8% with a predictor per
layer over 40 layers, 4: 7B Q4_0, 5: 70B neuron-sharded); explicit flags win.

A step is one sparse FFN layer (union -> gathered gate/up -> ReLU*up ->
gathered down) over one batch of B tokens.  Steps rotate over L distinct
layer copies (own weights, own Zipf(0.8) activity) so the weights read per
cycle exceed the 126 MB L2 several times: no step reads another step's
weights from L2.  Timing: CUDA events on the launching stream around exactly
K steps replayed from CUDA graphs, barrier + synchronize on both sides, max
over ranks; the K-step region is repeated and the median reported.

Under torchrun (WORLD_SIZE > 1) the layer's neurons are sharded across the
ranks (gate/up rows, W_down rows; one all-reduce of the [B][d] fp32
partial outputs per layer: NCCL's, or with --peer the library's one-shot
kernel over NVLink peer memory): strong scaling of the same layer, so N = 1 is
the single-GPU run.  --replicas runs independent copies instead.

The JSON line adds: e2e_bits (e2e with the sets as bit words instead of
fp32 labels), per_batch (the same layer at B = 1..32), dense_cublas
(the dense FFN through cuBLAS fp16 GEMMs with fp32 accumulation, same
config), device_error (the workspace's error word after every timed region;
non-zero fails the run), shard_parity / allreduce_us (the step's collective
alone) / nccl_allreduce_us when sharded.

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
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "sparse-FFN tokens/s per layer vs batch; % HBM roofline on active bytes"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0
PRED_RANK = 1024  # DejaVu predictor rank D (BASELINE configs 1 and 3)
SWEEP_BATCHES = (1, 2, 4, 8, 16, 32)


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", default="7b")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--activity", type=float, default=0.10)
    ap.add_argument("--path", choices=["auto", "gemv", "tensor"], default="auto")
    ap.add_argument("--per-token", type=int, default=1)
    ap.add_argument("--layers", type=int, default=0, help="distinct layer copies rotated (0 = auto)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-sweep", action="store_true", help="skip the per-batch curve")
    ap.add_argument("--no-dense", action="store_true", help="skip the cuBLAS dense comparator")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--repeats", type=int, default=0, help="timed K-step regions (0 = enough for ~0.3 s)")
    ap.add_argument("--shard", action="store_true", help="shard the layer's neurons across the ranks")
    ap.add_argument("--replicas", action="store_true", help="under torchrun: independent replicas, no sharding")
    ap.add_argument("--peer", action="store_true",
                    help="sharded: the library's one-shot peer-memory all-reduce instead of NCCL's")
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


def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as fh:
            return float(json.load(fh)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def pred_launches(B):
    """Kernels of this library that spb_predict launches for set words (top-k,
    no index list): one fused launch at B = 1; hidden, logit and two selects
    up to 16 tokens; above, x -> fp16, a histogram pass and two selects around
    two cuBLASLt GEMMs."""
    return 1 if B == 1 else 4


def workload_name(a, U, B=None):
    wt = {"f16": "fp16 weights", "q8_0": "Q8_0 weights", "q4_0": "Q4_0 weights"}[a.wtype]
    act = (f"{a.activity:.0%} per-token activity from the DejaVu predictor (top-k, run ahead of the layer)"
           if a.predictor else f"{a.activity:.0%} per-token activity Zipf(0.8)")
    return f"{a.model} sparse FFN layer (ReLU-gated SwiGLU), B={B or a.batch}, {wt}, {act}, union U~{U}"


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


class Clocks:
    """Samples SM clocks and throttle reasons in-process (NVML, every ~1 ms)
    while the timed region runs."""
    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.rows = []
        self.err = None

    def __enter__(self):
        self.stop = threading.Event()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
            self.max_sm = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception as e:  # noqa: BLE001
            self.err = f"nvml unavailable: {e}"
            return self

        def loop():
            while not self.stop.is_set():
                try:
                    sm = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                    rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                    self.rows.append((sm, rs))
                except Exception:  # noqa: BLE001
                    pass
                time.sleep(0.001)

        self.th = threading.Thread(target=loop, daemon=True)
        self.th.start()
        return self

    def __exit__(self, *exc):
        self.stop.set()
        if getattr(self, "th", None):
            self.th.join(timeout=2)

    def summary(self):
        if self.err or not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [self.err or "no samples"], "samples": 0}
        reasons = sorted({n for _, r in self.rows for n, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(s for s, _ in self.rows), "sm_max_mhz": self.max_sm,
                "reasons": reasons, "samples": len(self.rows), "source": "NVML in-process, ~1 ms"}


def layer_copies(a, bytes_per_layer):
    """Distinct layer copies so one rotation touches >= 3x the L2."""
    return a.layers or int(min(32, max(4, math.ceil(3 * L2_BYTES / bytes_per_layer))))


def rotation(a, d, f, ws_n, sharded):
    """Whether the per-batch curve runs, and the layer copies rotated: enough
    for the smallest batch timed (both arms use it, so their records match)."""
    from spbatch_b200.workload import active_bytes
    w_bytes = {"f16": 2.0, "q8_0": 34 / 32, "q4_0": 18 / 32}[a.wtype]
    pred_bytes = (d * PRED_RANK + PRED_RANK * (f // (ws_n if sharded else 1))) * 2 if a.predictor else 0
    sweep = (not a.no_sweep and ws_n == 1 and a.wtype == "f16" and not a.predictor and a.model == "7b"
             and a.batch == 32)
    Bs = sorted(set(SWEEP_BATCHES) | {a.batch}) if sweep else [a.batch]
    est_min = min(active_bytes(d, min(f, int(a.activity * f * min(B, 8))), B, w_bytes, pred_bytes) for B in Bs)
    if sharded:
        est_min /= ws_n
    return sweep, layer_copies(a, est_min)


def make_weights(a, L, d, f0, f1, device, seed):
    """L weight copies [f1 - f0][d] (this rank's rows) in the requested format."""
    import torch
    import spbatch_b200 as spb
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    out = []
    if a.wtype != "f16":
        # ggml block quantisation of one fp32 N(0, 0.02^2) set (host quantiser,
        # byte-identical to the oracle); every layer gets its own copy, so the
        # rotation still touches distinct addresses
        wt = spb.W_Q8_0 if a.wtype == "q8_0" else spb.W_Q4_0
        base = [torch.from_numpy(spb.quantize((torch.randn((f1 - f0, d), generator=gen, device=device) * 0.02)
                                              .cpu().numpy(), wt)).to(device) for _ in range(3)]
        return [[q.clone() for q in base] for _ in range(L)]
    for _ in range(L):
        out.append([(torch.randn((f1 - f0, d), generator=gen, device=device) * 0.02).half() for _ in range(3)])
    return out


def make_inputs(a, B, L, d, f, k, f0, f1, device, seed):
    """Per layer: x [B][d] and labels [B][f1 - f0] (this rank's columns), host and device."""
    import torch
    from spbatch_b200.workload import zipf_active_labels
    out = []
    for l in range(L):
        x_np = np.random.default_rng([seed, l, B]).standard_normal((B, d)).astype(np.float32)
        lab_full = zipf_active_labels(B, f, k, seed=seed, layer=l)
        lab_np = np.ascontiguousarray(lab_full[:, f0:f1])
        out.append(dict(i=l, x_np=x_np, lab_np=lab_np, lab_full=lab_full, x=torch.from_numpy(x_np).to(device),
                        lab=torch.from_numpy(lab_np).to(device), U=int((lab_np > 0).any(0).sum()),
                        U_full=int((lab_full > 0).any(0).sum()), out=torch.empty((B, d), device=device)))
    return out


class Timer:
    """K steps replayed from CUDA graphs on one stream, timed with CUDA events;
    the K-step region is repeated and the median per-step time kept."""

    def __init__(self, torch, stream, L, body, graphs=True):
        self.torch, self.stream, self.L, self.body = torch, stream, L, body
        self.graphs = graphs
        self.cache = {}

    def _graph(self, n):
        torch = self.torch
        if n not in self.cache:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self.stream):
                for i in range(n):
                    self.body(i % self.L)
            self.cache[n] = g
        return self.cache[n]

    def _run(self, K):
        full, rem = divmod(K, self.L)
        if self.graphs:
            gf = self._graph(self.L) if full else None
            gr = self._graph(rem) if rem else None
            for _ in range(full):
                gf.replay()
            if gr is not None:
                gr.replay()
        else:
            for i in range(K):
                self.body(i % self.L)

    def warm(self, W):
        torch = self.torch
        with torch.cuda.stream(self.stream):
            for i in range(max(3, W)):
                self.body(i % self.L)
            if self.graphs:  # capture (and run once) outside the timed region
                self._run(self.L + 1)
        torch.cuda.synchronize()

    def time(self, K, repeats, dist=None, device=None):
        torch = self.torch
        samples = []
        for _ in range(repeats):
            if dist is not None:
                dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(self.stream):
                e0.record(self.stream)
                self._run(K)
                e1.record(self.stream)
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            if dist is not None:
                t = torch.tensor([ms], device=device)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                ms = float(t.item())
            samples.append(ms / K)
        return statistics.median(samples), samples


def run_ours(a):
    import torch
    import spbatch_b200 as spb
    from spbatch_b200.shard import shard_range
    from spbatch_b200.workload import SHAPES, active_bytes

    ws_n, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = None
    if ws_n > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=device)
    sharded = ws_n > 1 and not a.replicas
    path = {"auto": spb.PATH_AUTO, "gemv": spb.PATH_GEMV, "tensor": spb.PATH_TENSOR}[a.path]
    wtype = {"f16": spb.W_F16, "q8_0": spb.W_Q8_0, "q4_0": spb.W_Q4_0}[a.wtype]
    w_bytes = {"f16": 2.0, "q8_0": 34 / 32, "q4_0": 18 / 32}[a.wtype]
    d, f = SHAPES[a.model]["d"], SHAPES[a.model]["f"]
    k = int(round(a.activity * f))
    f0, f1 = shard_range(f, ws_n, rank) if sharded else (0, f)
    seed = 0 if sharded else rank  # sharded: the same batch on every rank
    pred_bytes = (d * PRED_RANK + PRED_RANK * (f1 - f0)) * 2 if a.predictor else 0

    # layer copies: enough for the smallest batch the run times
    sweep, L = rotation(a, d, f, ws_n, sharded)
    Wl = make_weights(a, L, d, f0, f1, device, 1234 + (0 if sharded else rank))
    P = None
    pws = None
    if a.predictor:
        gen = torch.Generator(device=device)
        gen.manual_seed(99 + rank)
        # DejaVu low-rank predictor per layer: P1 [D][d] ~ N(0, 1/d), P2 [f][D] ~ N(0, 1/D)
        P = [[(torch.randn((PRED_RANK, d), generator=gen, device=device) / math.sqrt(d)).half(),
              (torch.randn((f1 - f0, PRED_RANK), generator=gen, device=device) / math.sqrt(PRED_RANK)).half()]
             for _ in range(L)]
    stream = torch.cuda.Stream(device)
    peak, peak_kind = hbm_peak()
    peer = None
    if sharded and a.peer:  # the exchange step through the library's all-reduce over NVLink peer memory
        from spbatch_b200.shard import PeerAllReduce
        peer = PeerAllReduce(max(SWEEP_BATCHES + (a.batch,)) * d, device)
    errors = []

    def measure(B, headline):
        layers = make_inputs(a, B, L, d, f, k, f0, f1, device, seed)
        ws = spb.new_workspace(B, d, f1 - f0, 0, device)
        pw = spb.predict_workspace(B, PRED_RANK, f1 - f0, device) if a.predictor else None
        if a.predictor:  # the predictor's own top-k labels drive each layer
            for ly in layers:
                spb.predict(P[ly["i"]][0], P[ly["i"]][1], ly["x"], k=k, out=ly["lab"], workspace=pw)
            torch.cuda.synchronize()
            for ly in layers:
                ly["lab_np"] = ly["lab"].cpu().numpy()
                ly["U"] = ly["U_full"] = int((ly["lab_np"] > 0).any(0).sum())
                # the timed step passes the sets as bit words (spb_predict ->
                # spb_ffn_forward_bits), no [B][f] label matrix in between
                ly["bits"] = torch.zeros((B, (f1 - f0 + 31) // 32), dtype=torch.int32, device=device)

        def fwd(i, x=None, lab=None, out=None):
            ly = layers[i]
            xx = ly["x"] if x is None else x
            ll = ly["lab"] if lab is None else lab
            o = ly["out"] if out is None else out
            # sharded with the peer all-reduce: the layer writes its partial
            # into the rank's mapped buffer, the reduction writes `o`
            po = peer.partial(B * d).view(B, d) if peer is not None else o
            if a.predictor:
                spb.predict(P[i][0], P[i][1], xx, k=k, bits_out=ly["bits"], labels=False, workspace=pw)
                spb.ffn_forward(*Wl[i], xx, bits=ly["bits"], f=f1 - f0, wtype=wtype, out=po,
                                per_token_mask=bool(a.per_token), path=path, workspace=ws)
            else:
                spb.ffn_forward(*Wl[i], xx, ll, wtype=wtype, out=po, per_token_mask=bool(a.per_token), path=path,
                                workspace=ws)
            if peer is not None:  # one all-reduce of the [B][d] partial outputs
                peer.reduce(B * d, o)
            elif sharded:
                dist.all_reduce(o)

        timer = Timer(torch, stream, L, fwd, graphs=True)
        timer.warm(a.warmup)
        K = a.steps if headline else min(a.steps, 2000)
        reps = a.repeats or max(3, min(25, int(0.3 / max(1e-6, K * 70e-6))))
        clk = Clocks(local) if headline else None
        if clk:
            with clk:
                ms, samples = timer.time(K, reps, dist, device)
        else:
            ms, samples = timer.time(K, reps, dist, device)
        err = spb.device_error(ws)
        Us = [ly["U"] for ly in layers]
        bytes_step = float(np.mean([active_bytes(d, U, B, w_bytes, pred_bytes) for U in Us]))
        res = dict(B=B, ms=ms, samples=samples, reps=reps, K=K, err=err, Us=Us, layers=layers, ws=ws, fwd=fwd,
                   bytes=bytes_step, timer=timer, clocks=clk.summary() if clk else None, pw=pw)
        errors.append(err)
        return res

    head = measure(a.batch, True)
    layers, ws = head["layers"], head["ws"]
    K = head["K"]
    ms = head["ms"]
    tokens_per_step = a.batch * (1 if sharded else ws_n)
    value = tokens_per_step / (ms / 1e3)
    achieved = head["bytes"] / (ms / 1e3) / 1e9

    # sharded: parity of the all-reduced output with the single-GPU layer
    shard_parity = None
    allreduce_us = None
    if sharded and a.wtype == "f16":
        o = torch.empty((a.batch, d), device=device)
        with torch.cuda.stream(stream):
            head["fwd"](0, out=o)
        torch.cuda.synchronize()
        ok = torch.tensor([1], device=device)
        if rank == 0:
            gen = torch.Generator(device=device)
            gen.manual_seed(1234)
            # rebuild the full layer 0 exactly as make_weights drew it, rank by rank
            parts = []
            for r in range(ws_n):
                r0, r1 = shard_range(f, ws_n, r)
                g2 = torch.Generator(device=device)
                g2.manual_seed(1234)
                parts.append([(torch.randn((r1 - r0, d), generator=g2, device=device) * 0.02).half()
                              for _ in range(3)])
            Wfull = [torch.cat([p[m] for p in parts]).contiguous() for m in range(3)]
            lab_full = torch.from_numpy(layers[0]["lab_full"]).to(device)
            ref = spb.ffn_forward(*Wfull, layers[0]["x"], lab_full, wtype=wtype, per_token_mask=bool(a.per_token),
                                  path=path, check=True)
            got, want = o.cpu().numpy().astype(np.float64), ref.cpu().numpy().astype(np.float64)
            bad = np.abs(got - want) > 1e-3 + 1e-2 * np.abs(want)
            good = bad.mean() <= (5e-4 if d >= 8192 else 0.0) and np.all(np.abs(got - want) <= 3e-3 + 1e-2 * np.abs(want))
            ok = torch.tensor([1 if good else 0], device=device)
            del Wfull, parts
        dist.broadcast(ok, 0)
        shard_parity = bool(ok.item())
    nccl_us = None
    if sharded:
        # the collective alone: 50 all-reduces of the [B][d] fp32 output
        # captured in one graph, replayed on the compute stream -- the one the
        # step uses, and NCCL's for comparison
        buf = torch.zeros((a.batch, d), device=device)
        art = Timer(torch, stream, 1, lambda i: dist.all_reduce(buf), graphs=True)
        art.warm(3)
        nccl_us = art.time(50, 5, dist, device)[0] * 1e3
        allreduce_us = nccl_us
        if peer is not None:
            n = a.batch * d
            prt = Timer(torch, stream, 1, lambda i: peer.reduce(n, buf), graphs=True)
            prt.warm(3)
            allreduce_us = prt.time(50, 5, dist, device)[0] * 1e3
            if peer.error():
                errors.append(100 + peer.error())

    # e2e: pinned host inputs copied in and the output copied back every step
    pinned = [dict(x=torch.from_numpy(ly["x_np"]).pin_memory(), lab=torch.from_numpy(ly["lab_np"]).pin_memory(),
                   out=torch.empty((a.batch, d)).pin_memory()) for ly in layers]
    xin = [torch.empty_like(ly["x"]) for ly in layers]
    labin = [torch.empty_like(ly["lab"]) for ly in layers]

    def e2e_body(i):
        xin[i].copy_(pinned[i]["x"], non_blocking=True)
        if not a.predictor:  # with the predictor the labels are produced on the device from x
            labin[i].copy_(pinned[i]["lab"], non_blocking=True)
        head["fwd"](i, x=xin[i], lab=labin[i], out=layers[i]["out"])
        pinned[i]["out"].copy_(layers[i]["out"], non_blocking=True)

    etimer = Timer(torch, stream, L, e2e_body, graphs=True)
    etimer.warm(3)
    ms_e2e, _ = etimer.time(K, max(3, head["reps"] // 2), dist, device)
    errors.append(spb.device_error(ws))

    # the same end to end with the sets as bit words (spb_ffn_forward_bits:
    # 1/32 of the label bytes cross PCIe), single GPU without the predictor
    e2e_bits = None
    if not a.predictor and not sharded:
        W = (f + 31) // 32

        def words(lab):
            b = np.packbits(lab > 0, axis=1, bitorder="little")
            b = np.pad(b, ((0, 0), (0, 4 * W - b.shape[1])))
            return torch.from_numpy(np.ascontiguousarray(b).view(np.int32)).pin_memory()

        pbits = [words(ly["lab_np"]) for ly in layers]
        bitsin = [torch.empty((a.batch, W), dtype=torch.int32, device=device) for _ in layers]

        def e2e_bits_body(i):
            xin[i].copy_(pinned[i]["x"], non_blocking=True)
            bitsin[i].copy_(pbits[i], non_blocking=True)
            spb.ffn_forward(*Wl[i], xin[i], bits=bitsin[i], f=f, wtype=wtype, out=layers[i]["out"],
                            per_token_mask=bool(a.per_token), path=path, workspace=ws)
            pinned[i]["out"].copy_(layers[i]["out"], non_blocking=True)

        btimer = Timer(torch, stream, L, e2e_bits_body, graphs=True)
        btimer.warm(3)
        ms_b, _ = btimer.time(K, max(3, head["reps"] // 2), dist, device)
        errors.append(spb.device_error(ws))
        e2e_bits = {"value": tokens_per_step / (ms_b / 1e3), "unit": "tokens/s", "ms_per_step": ms_b,
                    "h2d_bytes_per_step": a.batch * d * 4 + a.batch * W * 4, "d2h_bytes_per_step": a.batch * d * 4,
                    "sets": "bit words [B][ceil(f/32)] (spb_ffn_forward_bits)"}

    rec = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws_n, "steps": K, "warmup": a.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong" if sharded else "weak",
        "vs_baseline": None, "dtype": a.wtype,
        "data": "synthetic (seeded N(0,0.02^2) weights, N(0,1) x, Zipf(0.8) activity; no dataset)",
        "config": config_dict(a, d, f, f1 - f0, k, head["Us"], [ly["U_full"] for ly in layers], L,
                              head["bytes"], ws_n, sharded),
        "roofline": {"bound": "hbm", "kernel": "whole layer (every launch of the step)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} hbm_gbs", "traffic": traffic_from_profiles(a),
                     "bytes_per_step": head["bytes"]},
        "e2e": {"value": tokens_per_step / (ms_e2e / 1e3), "unit": "tokens/s",
                "h2d_bytes_per_step": a.batch * d * 4 + (0 if a.predictor else a.batch * (f1 - f0) * 4),
                "d2h_bytes_per_step": a.batch * d * 4, "ms_per_step": ms_e2e},
        "e2e_bits": e2e_bits,
        "clocks": head["clocks"],
        "timing": {"repeats": head["reps"], "ms_per_step_samples": [round(s, 5) for s in head["samples"]],
                   "statistic": "median over repeats of the K-step region"},
        "gpu_launches": int(spb.lib().spb_ffn_launches(a.batch, d, wtype, path) + (pred_launches(a.batch) if a.predictor else 0)) * K,
    }
    if sharded:
        rec["shard_parity"] = shard_parity
        rec["allreduce_us"] = allreduce_us
        rec["nccl_allreduce_us"] = nccl_us
        rec["collective"] = ("one-shot all-reduce over NVLink peer memory (spb_allreduce_peer, own kernel)"
                             if peer is not None else "NCCL all-reduce")
        rec["parallelism"] = f"neuron-sharded tp{ws_n}"

    if sweep:
        per = {}
        for B in SWEEP_BATCHES:
            if B == a.batch:
                r = head
            else:
                r = measure(B, False)
            ach = r["bytes"] / (r["ms"] / 1e3) / 1e9
            per[str(B)] = {"tokens_per_s": B / (r["ms"] / 1e3), "us_per_step": r["ms"] * 1e3,
                           "union_mean": float(np.mean(r["Us"])), "achieved_gbs": ach, "frac": ach / peak,
                           "device_error": r["err"]}
            if B != a.batch:
                del r
                torch.cuda.empty_cache()
        rec["per_batch"] = per

    if not a.no_dense and ws_n == 1 and a.wtype == "f16" and not a.predictor:
        rec["dense_cublas"] = dense_comparator(a, Wl, layers, stream, K, d, f, peak)

    rec["device_error"] = max(errors) if errors else 0
    if rank == 0 and ws_n == 1 and not a.no_cpu:
        rec["cpu_baseline"] = cpu_baseline(a, layers[0], Wl[0], budget=a.cpu_budget)
    if rank == 0:
        print(json.dumps(rec), flush=True)
    code = 0
    if rec["device_error"]:
        print(f"device error word {rec['device_error']}: a bounded device wait ran out; the run is invalid",
              file=sys.stderr, flush=True)
        code = 1
    if ws_n > 1:
        # All work is done and the line is printed.  CUDA graphs that captured
        # NCCL calls are still alive here, and tearing the process group down
        # under them can block; every rank leaves after a final barrier.
        torch.cuda.synchronize()
        dist.barrier()
        sys.stdout.flush()
        sys.stderr.flush()
        os._exit(code)
    if code:
        sys.exit(code)


def config_dict(a, d, f, f_shard, k, Us, Us_full, L, bytes_step, ws_n, sharded):
    """The workload description shared by both arms."""
    return {"workload": workload_name(a, int(np.mean(Us_full))), "d": d, "f": f, "f_per_gpu": f_shard,
            "batch": a.batch, "k_per_token": k, "union_mean": float(np.mean(Us_full)), "layers_rotated": L,
            "per_token_mask": bool(a.per_token), "path": a.path, "weights": a.wtype,
            "predictor": (f"DejaVu rank {PRED_RANK}, top-{k} per token, run ahead of every layer"
                          if a.predictor else None),
            "l2": f"inputs larger than L2: {L} layer copies rotated, "
                  f"{L * bytes_step / 1e6:.0f} MB touched per cycle vs 126 MB L2",
            "parallelism": (f"neuron-sharded tp{ws_n} + one all-reduce" if sharded else
                            f"replicas x{ws_n}" if ws_n > 1 else "single GPU")}


def dense_comparator(a, Wl, layers, stream, K, d, f, peak):
    """The dense FFN through cuBLAS (torch fp16 GEMMs, fp32 accumulation and
    no reduced-precision reductions), rotating over the same layer copies."""
    import torch
    torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction = False
    L = len(Wl)
    x16 = [ly["x"].half() for ly in layers]
    outs = [torch.empty((a.batch, d), dtype=torch.float16, device=ly["x"].device) for ly in layers]

    def body(i):
        wg, wu, wd = Wl[i]
        g = x16[i] @ wg.T
        u = x16[i] @ wu.T
        h = torch.relu(g) * u
        torch.matmul(h, wd, out=outs[i])

    t = Timer(torch, stream, L, body, graphs=True)
    t.warm(3)
    ms, _ = t.time(min(K, 2000), 5)
    dense_bytes = 3.0 * d * f * 2 + a.batch * d * 4
    ach = dense_bytes / (ms / 1e3) / 1e9
    return {"tokens_per_s": a.batch / (ms / 1e3), "us_per_step": ms * 1e3, "achieved_gbs": ach,
            "frac_of_peak": ach / peak, "bytes_per_step": dense_bytes,
            "what": "dense FFN (all f neurons), cuBLAS fp16 GEMMs with fp32 accumulation via torch.matmul, "
                    "graph-replayed over the same rotated layer copies"}


def traffic_from_profiles(a):
    """DRAM bytes per layer from the committed ncu summary, when one exists for this workload."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as fh:
            t = json.load(fh)
        return t.get(f"{a.model}_b{a.batch}_{a.path}")
    except Exception:
        return None


def _cpu_ffn():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    from cpu_ffn import MaskedDenseFFN, time_steps
    return MaskedDenseFFN, time_steps


def cpu_baseline(a, ly, W, budget=15.0):
    MaskedDenseFFN, time_steps = _cpu_ffn()
    if a.wtype == "f16":
        Wn = [w.float().cpu().numpy() for w in W]
    else:  # the CPU baseline computes with the dequantised weights (oracle dequantisation)
        import oracle
        qt = 8 if a.wtype == "q8_0" else 4
        d = ly["x_np"].shape[1]
        Wn = [oracle.dequantize(w.cpu().numpy(), qt, d) for w in W]
    ffn = MaskedDenseFFN(*Wn)
    n, s = time_steps(ffn, ly["x_np"], ly["lab_np"], budget_s=budget)
    return {"value": a.batch * n / s, "unit": "tokens/s", "cores": ffn.threads, "kind": "port",
            "sample": f"{n} whole steps (one {a.model} layer, B={a.batch}) in {s:.1f} s, PyTorch fp32 "
                      f"masked-dense FFN on {ffn.threads} host threads"}


def run_reference(a):
    """The reference's CPU path on the same workload: the same layers' x and
    labels (same seeds as the GPU arm, rotated the same way), the same
    warm-up count, and the same config record."""
    ws_n, rank, _ = dist_env()
    if rank != 0:
        return
    import torch
    from spbatch_b200.workload import SHAPES, active_bytes, zipf_active_labels
    d, f = SHAPES[a.model]["d"], SHAPES[a.model]["f"]
    k = int(round(a.activity * f))
    _, L = rotation(a, d, f, ws_n, ws_n > 1 and not a.replicas)
    g = torch.Generator().manual_seed(1234)
    # one fp16-valued weight set: the dense CPU path's cost does not depend on the values
    W = [(torch.randn((f, d), generator=g) * 0.02).half().float().numpy() for _ in range(3)]
    labs = [zipf_active_labels(a.batch, f, k, seed=0, layer=l) for l in range(L)]
    xs = [np.random.default_rng([0, l, a.batch]).standard_normal((a.batch, d)).astype(np.float32) for l in range(L)]
    Us = [int((lab > 0).any(0).sum()) for lab in labs]
    MaskedDenseFFN, _ = _cpu_ffn()
    ffn = MaskedDenseFFN(*W)
    for i in range(a.warmup):
        ffn(xs[i % L], labs[i % L])
    budget = min(120.0, max(10.0, a.cpu_budget * 4))
    n = 0
    t0 = time.perf_counter()
    while n < a.steps and (n < 3 or time.perf_counter() - t0 < budget):
        ffn(xs[n % L], labs[n % L])
        n += 1
    s = time.perf_counter() - t0
    value = a.batch * n / s
    a2 = argparse.Namespace(**vars(a))
    rec = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": ws_n, "steps": n,
        "warmup": a.warmup, "ms_per_step": s / n * 1e3, "higher_is_better": True,
        "scaling": "strong" if ws_n > 1 and not a.replicas else "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (the GPU arm's seeds)",
        "config": config_dict(a2, d, f, f, k, Us, Us, L, float(np.mean([active_bytes(d, U, a.batch) for U in Us])),
                              ws_n, ws_n > 1 and not a.replicas),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": ffn.threads, "kind": "port",
                         "sample": f"{n} of the requested {a.steps} steps (time-bounded, {budget:.0f} s), the "
                                   f"GPU arm's {L} rotated batches, PyTorch fp32 masked-dense FFN restating "
                                   f"MLP_naive on {ffn.threads} host threads"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(rec), flush=True)


def main():
    a = parse()
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
