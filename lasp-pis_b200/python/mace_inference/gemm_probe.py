"""Run the engine's tensor-core GEMM (tc_gemm, through mace_debug_gemm) on one node-linear
shape, for kernel captures:  python -m mace_inference.gemm_probe --m 10000 --n 512 --k 512 --batch 7

The default shape is the heaviest MH1 node linear at C3: linear_2 of layer 0, its l = 3 path
(512 -> 512 channels, 7 components, 10,000 nodes).  Each call splits the weights on the host,
so only the kernel itself is meaningful to a profiler.
"""
import argparse
import ctypes as ct

from .library import library_path


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--m", type=int, default=10000)
    ap.add_argument("--n", type=int, default=512)
    ap.add_argument("--k", type=int, default=512)
    ap.add_argument("--batch", type=int, default=7)
    ap.add_argument("--calls", type=int, default=3)
    ap.add_argument("--library", default=None)
    args = ap.parse_args()
    import torch
    lib = ct.CDLL(str(args.library or library_path()))
    lib.mace_debug_gemm.argtypes = [ct.c_int] * 4 + [ct.c_void_p] * 3 + [ct.c_int, ct.c_int]
    lib.mace_last_error.restype = ct.c_char_p
    g = torch.Generator(device="cuda").manual_seed(1)
    A = torch.randn(args.batch, args.m, args.k, device="cuda", generator=g)
    B = torch.randn(args.k, args.n, device="cuda", generator=g) / args.k ** 0.5
    C = torch.empty(args.batch, args.m, args.n, device="cuda")
    for _ in range(args.calls):
        if lib.mace_debug_gemm(args.m, args.n, args.k, args.batch, A.data_ptr(), B.data_ptr(), C.data_ptr(), 0, 1):
            raise SystemExit(lib.mace_last_error().decode())
    torch.cuda.synchronize()
    print(f"tc_gemm {args.m}x{args.n}x{args.k} batch {args.batch}: {args.calls} calls ok")


if __name__ == "__main__":
    main()
