"""Fixed, seeded workloads for profilers (ncu), one per product kernel.

    python tests/tools/capture.py KIND [B] [model]

KIND: tensor | stream | gemv | union | predict | dropin | dequant | bits.
Each kind runs a few warm-up calls and then `calls` more, on the model's
layer shape (7B by default: d = 4096, f = 11008) with 10% Zipf(0.8)
activity per token and fp16 N(0, 0.02^2) weights, four layer copies
rotated.  Device memory stays near 1-2 GB, so a capture with `ncu -k
regex:<kernel> -s <warm-up launches> -c <n>` ends in seconds.  The
profiles/ summaries name the exact command they ran.
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)


def main(argv):
    import numpy as np
    import torch
    import spbatch_b200 as spb
    from spbatch_b200.workload import SHAPES, zipf_active_labels
    kind = argv[1]
    B = int(argv[2]) if len(argv) > 2 else 32
    model = argv[3] if len(argv) > 3 else "7b"
    d, f = SHAPES[model]["d"], SHAPES[model]["f"]
    k = f // 10
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    L, calls = 4, 8
    labs = [torch.from_numpy(zipf_active_labels(B, f, k, seed=0, layer=l)).to(dev) for l in range(L)]
    x = torch.randn((B, d), generator=g, device=dev)
    if kind in ("tensor", "stream", "gemv", "bits", "dropin"):
        W = [[(torch.randn((f, d), generator=g, device=dev) * 0.02).half() for _ in range(3)] for _ in range(L)]
    if kind in ("tensor", "stream", "gemv", "bits"):
        path = {"tensor": spb.PATH_TENSOR, "stream": spb.PATH_GEMV, "gemv": spb.PATH_GEMV, "bits": spb.PATH_AUTO}[kind]
        ws = spb.new_workspace(B, d, f, 0, dev)
        out = torch.empty((B, d), device=dev)
        # gemv: index outputs requested, which the fallback GEMV serves for B > 4
        merge = torch.empty(f, dtype=torch.int32, device=dev) if kind == "gemv" else None
        cnt = torch.empty(1, dtype=torch.int32, device=dev) if kind == "gemv" else None
        if kind == "bits":
            bits = []
            for lab in labs:
                b = np.packbits((lab.cpu().numpy() > 0).astype(np.uint8), axis=1, bitorder="little")
                b = np.pad(b, ((0, 0), (0, (-b.shape[1]) % 4)))
                bits.append(torch.from_numpy(np.ascontiguousarray(b.view(np.int32))).to(dev))
        for it in range(calls):
            l = it % L
            kw = dict(bits=bits[l], f=f) if kind == "bits" else dict(idx=labs[l])
            spb.ffn_forward(*W[l], x, **kw, workspace=ws, out=out, path=path, merge_idx_out=merge, count_out=cnt,
                            per_token_mask=kind != "gemv")
    elif kind == "union":
        ws = spb.new_workspace(B, 64, f, 8, dev)
        for it in range(calls):
            spb.union(labs[it % L], group=8, workspace=ws)
    elif kind == "predict":
        D = 1024
        P1 = [(torch.randn((D, d), generator=g, device=dev) / d ** 0.5).half() for _ in range(L)]
        P2 = [(torch.randn((f, D), generator=g, device=dev) / D ** 0.5).half() for _ in range(L)]
        pws = spb.predict_workspace(B, D, f, dev)
        out = torch.empty((B, f), device=dev)
        for it in range(calls):
            spb.predict(P1[it % L], P2[it % L], x, k=k, out=out, workspace=pws)
    elif kind == "dropin":
        # the reference's MLP_BS composition through the drop-in API (groups of 8)
        M, N, K = f, B, d
        S = (B + 7) // 8
        merge = torch.zeros((S, f), dtype=torch.int32, device=dev)
        act = torch.zeros(S, dtype=torch.int32, device=dev)
        dst = [torch.zeros((B, f), device=dev) for _ in range(4)]
        outd = torch.zeros((B, d), device=dev)
        st = torch.cuda.current_stream().cuda_stream
        get_idx = spb.dropin.fn("get_idx_cuda")
        gate_up = spb.dropin.fn("gate_and_up_mul_mat_cuda_sparse")
        relu_mul = spb.dropin.fn("relu_and_mul_cuda")
        down = spb.dropin.fn("down_mul_mat_cuda_sparse")
        for it in range(calls):
            wg, wu, wd = W[it % L]
            get_idx(labs[it % L].data_ptr(), merge.data_ptr(), act.data_ptr(), B, f, st)
            gate_up(wg.data_ptr(), wu.data_ptr(), x.data_ptr(), dst[0].data_ptr(), dst[1].data_ptr(), merge.data_ptr(),
                    M, N, K, act.data_ptr(), st, st)
            relu_mul(dst[0].data_ptr(), dst[1].data_ptr(), dst[3].data_ptr(), M, N, st)
            # cuda/ffn_test.cu: down_mul_mat_cuda_sparse(w, h, out, merge, K = d, M = batch, N = f, ...)
            down(wd.data_ptr(), dst[3].data_ptr(), outd.data_ptr(), merge.data_ptr(), K, N, M, act.data_ptr(), st)
    elif kind == "dequant":
        rb = int(spb.lib().spb_weight_row_bytes(spb.W_Q4_0, d))
        q = torch.randint(0, 255, (f, rb), dtype=torch.uint8, device=dev)
        q[:, rb - d // 16:] = 0  # scales 0.0: finite output
        outq = torch.empty((f, d), device=dev)
        for it in range(calls):
            assert spb.lib().spb_dequantize_rows(q.data_ptr(), spb.W_Q4_0, f, d, outq.data_ptr(),
                                                 torch.cuda.current_stream().cuda_stream) == 0
    else:
        raise SystemExit(f"unknown kind {kind}")
    torch.cuda.synchronize()
    print("ok", kind, B, model)


if __name__ == "__main__":
    main(sys.argv)
