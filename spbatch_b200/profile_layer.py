"""A fixed workload for profilers: four seeded 7B layers (fp16 weights,
10% Zipf(0.8) activity per token), one spb_ffn_forward per layer in turn,
eight calls.  Run it under ncu with -k/-s/-c to capture one launch:

    python -m spbatch_b200.profile_layer B [tensor|gemv|auto]
"""
import sys


def main(argv):
    import torch
    import spbatch_b200 as spb
    from spbatch_b200.workload import SHAPES, zipf_active_labels
    B = int(argv[1]) if len(argv) > 1 else 32
    path = {"tensor": spb.PATH_TENSOR, "gemv": spb.PATH_GEMV, "auto": spb.PATH_AUTO}[argv[2] if len(argv) > 2 else "auto"]
    d, f = SHAPES["7b"]["d"], SHAPES["7b"]["f"]
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev)
    g.manual_seed(0)
    L = 4
    W = [[(torch.randn((f, d), generator=g, device=dev) * 0.02).half() for _ in range(3)] for _ in range(L)]
    labs = [torch.from_numpy(zipf_active_labels(B, f, 1101, seed=0, layer=l)).to(dev) for l in range(L)]
    x = torch.randn((B, d), generator=g, device=dev)
    ws = spb.new_workspace(B, d, f, 0, dev)
    out = torch.empty((B, d), device=dev)
    for it in range(8):
        spb.ffn_forward(*W[it % L], x, labs[it % L], workspace=ws, out=out, path=path)
    torch.cuda.synchronize()
    print("ok")


if __name__ == "__main__":
    main(sys.argv)
