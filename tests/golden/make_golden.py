"""Generates the golden fixtures of tests/golden/ by running the REFERENCE
kernel (blackwell_nvfp4_gemv.cu, built from its own source into oracle/_ref by
oracle/build_ref.py) on a GPU.

    python tests/golden/make_golden.py [out_dir]     (default: next to this script)

Fixtures (npz, inputs included so the CPU tests need no generator):
  kat_e2m1.npz  M=32 K=512 L=16: row m's first 16-element block holds code m%16,
                batch l's vector holds code l there, all scales 1.0, everything
                else zero -> c[m, l] = 16 * e2m1(m%16) * e2m1(l): the full
                16 x 16 product table of the reference's e2m1 decode.
  kat_e4m3.npz  M=256 K=512 L=1: row m's first block holds code 1.0 with scale
                byte m, the vector is 1.0 with scale 1.0 -> c[m] = 16 * e4m3(m):
                all 256 e4m3 scale bytes through the reference's decode.
  config0.npz   M=256 K=1024 L=1 seeded inputs (seed 0) and the reference's c.
"""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def run_ref(ref, a, b, sfa, sfb, M, K, L):
    dev = torch.device("cuda")
    # an explicit [L, rows, cols] copy: numpy keeps odd strides on size-1 dims,
    # and the reference encodes the L stride even when L == 1
    perm = lambda t: torch.from_numpy(t.transpose(2, 0, 1).copy(order="C")).contiguous().to(dev).permute(1, 2, 0)
    c = torch.empty((L, 1, M), dtype=torch.float16, device=dev).permute(2, 1, 0)
    ref.nvfp4_gemv_forward(perm(a), perm(b), perm(sfa), perm(sfb), c, M, K, L)
    torch.cuda.synchronize()
    return c.cpu().numpy()


def main(out):
    import build_ref
    import __graft_entry__
    ref = build_ref.load()
    pkg = __graft_entry__.load_package()
    os.makedirs(out, exist_ok=True)

    M, K, L = 32, 512, 16
    a = np.zeros((M, K // 2, L), np.uint8)
    b = np.zeros((1, K // 2, L), np.uint8)
    for m in range(M):
        a[m, :8, :] = (m % 16) | ((m % 16) << 4)
    for l in range(L):
        b[0, :8, l] = l | (l << 4)
    sfa = np.full((M, K // 16, L), 0x38, np.uint8)
    sfb = np.full((1, K // 16, L), 0x38, np.uint8)
    np.savez(os.path.join(out, "kat_e2m1.npz"), a=a, b=b, sfa=sfa, sfb=sfb,
             c=run_ref(ref, a, b, sfa, sfb, M, K, L), shape=(M, K, L))

    M, K, L = 256, 512, 1
    a = np.zeros((M, K // 2, L), np.uint8)
    a[:, :8, :] = 0x22
    b = np.full((1, K // 2, L), 0x22, np.uint8)
    sfa = np.full((M, K // 16, L), 0x38, np.uint8)
    sfa[:, 0, 0] = np.arange(256, dtype=np.uint8)
    sfb = np.full((1, K // 16, L), 0x38, np.uint8)
    np.savez(os.path.join(out, "kat_e4m3.npz"), a=a, b=b, sfa=sfa, sfb=sfb,
             c=run_ref(ref, a, b, sfa, sfb, M, K, L), shape=(M, K, L))

    M, K, L = 256, 1024, 1
    x = pkg.inputs.gemv_inputs(M, K, L, seed=0)
    arrs = [t.numpy() for t in (x.a, x.b, x.sfa, x.sfb)]
    np.savez(os.path.join(out, "config0.npz"), a=arrs[0], b=arrs[1], sfa=arrs[2], sfb=arrs[3],
             c=run_ref(ref, *arrs, M, K, L), shape=(M, K, L))
    print("golden written to", out)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__)))
