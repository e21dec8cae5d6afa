"""Phase timeline of the tensor-core FFN kernel from its own %globaltimer
stamps (spb_trace_enable), for the kernel ncu cannot profile.

    python tests/tools/trace_tc.py [model] [B] [--bits] [--wtype q8|q4]

Runs the layer a few times on the model's shape (7B by default: d = 4096,
f = 11008) with 10% Zipf(0.8) activity, four layer copies rotated, traces two
consecutive launches and prints, per phase stamp, the min / median / max over
the CTAs (µs from the earliest CTA start), the gap between the two launches,
and the per-stage stamps of CTA 0.  Stamps: start (after the dependency
wait), phase0 / barrier / scan / emit_gu (prologue), scanned (first copy may
issue), gu_issued (last gate/up copy issued), gu_acc / xchg / h_done (first
accumulator, first pair exchange, last h published), first_flag (first down
h tile available), dn_issued / dn_acc (down copies issued / accumulator
ready), end.
"""
import argparse
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

NAMES = ["start", "scanned", "gu_issued", "gu_mma", "gu_acc", "xchg", "h_done", "first_flag", "dn_issued",
         "dn_acc", "end", "phase0", "barrier", "scan", "emit_gu", "emit_dn"]
SLOTS, CTAS = 16, 160
UNIT_BASE, STAGE_BASE = CTAS * SLOTS, CTAS * SLOTS + 128 * 4


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("model", nargs="?", default="7b")
    ap.add_argument("B", nargs="?", type=int, default=32)
    ap.add_argument("--bits", action="store_true", help="pass the sets as bit words")
    ap.add_argument("--wtype", choices=["f16", "q8", "q4"], default="f16")
    a = ap.parse_args()
    import numpy as np
    import torch
    import spbatch_b200 as spb
    from spbatch_b200.workload import SHAPES, zipf_active_labels
    d, f = SHAPES[a.model]["d"], SHAPES[a.model]["f"]
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    wt = {"f16": spb.W_F16, "q8": spb.W_Q8_0, "q4": spb.W_Q4_0}[a.wtype]
    layers = []
    qbase = None
    for l in range(4):
        if wt == spb.W_F16:
            W = [(torch.randn((f, d), generator=g, device=dev) * 0.02).half() for _ in range(3)]
        else:
            if qbase is None:
                qbase = [torch.from_numpy(spb.quantize((torch.randn((f, d), generator=g, device=dev) * 0.02)
                                                       .cpu().numpy(), wt)).to(dev) for _ in range(3)]
            W = [q.clone() for q in qbase]
        lab = zipf_active_labels(a.B, f, int(0.1 * f), seed=0, layer=l)
        b = np.packbits((lab > 0).astype(np.uint8), axis=1, bitorder="little")
        b = np.pad(b, ((0, 0), (0, (-b.shape[1]) % 4)))
        layers.append((W, torch.randn((a.B, d), generator=g, device=dev), torch.from_numpy(lab).to(dev),
                       torch.from_numpy(np.ascontiguousarray(b.view(np.int32))).to(dev)))
    ws = spb.new_workspace(a.B, d, f, 0, dev)
    n = STAGE_BASE + 256 * 4
    tr = [torch.zeros(n, dtype=torch.int64, device=dev) for _ in range(2)]
    for it in range(7):
        W, x, lab, bits = layers[it % 4]
        if it == 5:
            torch.cuda.synchronize()
        if it >= 5:
            spb.lib().spb_trace_enable(tr[it - 5].data_ptr(), n)
        sets = dict(bits=bits, f=f) if a.bits else dict(idx=lab)
        spb.ffn_forward(*W, x, **sets, wtype=wt, workspace=ws, path=spb.PATH_TENSOR)
    torch.cuda.synchronize()
    spb.lib().spb_trace_enable(None, 0)
    print("device error", spb.device_error(ws))
    t1 = tr[0].cpu().numpy()[:UNIT_BASE].reshape(CTAS, SLOTS).astype(np.float64)
    t2 = tr[1].cpu().numpy()[:UNIT_BASE].reshape(CTAS, SLOTS).astype(np.float64)
    print(f"gap between launches (last CTA end -> first CTA start): "
          f"{(t2[t2[:, 0] > 0, 0].min() - t1[t1[:, 10] > 0, 10].max()) / 1e3:.1f} us")
    t = t1[t1[:, 0] > 0]
    t0 = t[:, 0].min()
    for i, name in enumerate(NAMES):
        col = (t[:, i][t[:, i] > 0] - t0) / 1e3
        if len(col):
            print(f"{name:10s} min {col.min():7.1f} med {np.median(col):7.1f} max {col.max():7.1f} us (n={len(col)})")
    st = tr[0].cpu().numpy()[STAGE_BASE:STAGE_BASE + 1024].reshape(256, 4).astype(np.float64)
    rows = [i for i in range(256) if st[i].max() > 0]
    print("CTA 0 stage stamps (us): [0] issue / expansion start, [1] issued / arrived, [2] MMA saw it full")
    for i in rows[::max(1, len(rows) // 16)]:
        print(f"{i:4d} " + " ".join(f"{(v - t0) / 1e3:7.1f}" if v > 0 else "    nan" for v in st[i, :3]))


if __name__ == "__main__":
    main()
