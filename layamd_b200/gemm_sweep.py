"""Isolated encoder-GEMM sweep (benchmark configuration C5) on the engine's tcgen05 GEMM.

For M (packed tokens) in {512, 4096, 32768, 131072} and (K, N) in {(1024,3072), (1024,1024),
(1024,5248), (2624,1024)} -- the Wqkv, Wo, Wi and MLP-out projections of ModernBERT-large -- times the
kernel through the C ABI entry point ``laya_b200_gemm`` with CUDA events (warm-up, then `iters` back to
back launches on one stream), in bf16 (one bf16 product, fp32 accumulation) and in fp32-parity mode
(three bf16 products on hi/lo splits). Inputs: A ~ N(0,1), W ~ N(0,0.02), seed 5. Reports TFLOP/s
(2MNK/t, parity mode counted as the same 2MNK), the fraction of the measured sustained and burst bf16
peaks, the engine's plan for the shape (tile and K split; split shapes run through
``laya_b200_gemm_splitk``), torch.matmul (cuBLAS) on the same bf16 operands as a
comparator, and max|C - C_ref| / max|C_ref| against an fp64 reference GEMM of the fp32 inputs. The
bf16 rows write fp32 for that check; ``--no-check`` writes bf16 as cuBLAS does (like-for-like timing).

Usage: python -m layamd_b200.gemm_sweep [--m 512,4096] [--kn 1024x3072,...] [--epi store|geglu|rope|resid]
       [--modes bf16,parity] [--tile auto|128|256|pair] [--iters 20] [--no-check] [--json]
       python -m layamd_b200.gemm_sweep --sustained 3    # the C2 pass's GEMMs at the power cap vs cuBLAS
"""
import argparse
import ctypes
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EPI = {"store": 0, "rope": 1, "geglu": 2, "resid": 3}
TILES = {"128": 128, "256": 256, "pair": 512}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops_sustained"]), float(p["bf16_tflops"])
    except Exception:
        return 1400.0, 1590.0


def plan(L, M, N, K, sms, parity):
    """The engine's plan for this shape (laya_plan_gemm): the tile (the CTA-pair 256 x 256 tile when
    its tiles fill every co-resident pair twice, else the width with fewer whole waves) and the K
    split (slices for a few hundred rows of long K, where 128 x 128 tiles cannot fill the GPU)."""
    bn, splits = ctypes.c_int(0), ctypes.c_int(0)
    assert L.laya_plan_gemm(M, N, K, parity, sms, sms // 2, 0, ctypes.byref(bn), ctypes.byref(splits)) == 0
    return bn.value, splits.value


def interleave_geglu(W, I):
    import torch
    parts = []
    for j in range(0, I, 64):
        parts.append(W[j:j + 64])
        parts.append(W[I + j:I + j + 64])
    return torch.cat(parts).contiguous()


def sustained(L, seconds, rows=52287):
    """The C2 pass's four encoder GEMMs (QKV, attention-out, MLP-in, MLP-out at `rows` rows) run back
    to back for `seconds` each way, so that the GPU settles at its power cap as inside a long pass:
    cuBLAS (torch.matmul, bf16 output), this library with a plain bf16 store, and this library with the
    pass's fused epilogues (RoPE on QKV, fp32 residual add on the two residual GEMMs, GeGLU on MLP-in).
    Prints one line per run: ms per set of four and TFLOP/s (2MNK summed over the four)."""
    import time
    import torch
    shapes = [(1024, 3072), (1024, 1024), (1024, 5248), (2624, 1024)]  # (K, N)
    M = rows
    g = torch.Generator(device="cuda").manual_seed(5)
    A = {K: torch.randn(M, K, device="cuda", generator=g).bfloat16() for K in (1024, 2624)}
    W = [(0.02 * torch.randn(N, K, device="cuda", generator=g)).bfloat16() for K, N in shapes]
    O = [torch.empty(M, N, device="cuda", dtype=torch.bfloat16) for K, N in shapes]
    x = torch.zeros(M, 1024, device="cuda")
    pos = torch.randint(0, 512, (M,), device="cuda", dtype=torch.int32, generator=g)
    cs = torch.rand(512, 32, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    flops = sum(2.0 * M * N * K for K, N in shapes)
    vp = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    sms = torch.cuda.get_device_properties(0).multi_processor_count

    def ours(fused):
        for i, (K, N) in enumerate(shapes):
            epi, out, res = ((1, O[i], None), (3, None, x), (2, O[i], None), (3, None, x))[i] if fused else (0, O[i], None)
            bn, _ = plan(L, M, N, K, sms, False)
            rc = L.laya_b200_gemm(vp(A[K]), vp(W[i]), vp(out), vp(res), None, M, N, K, 1, epi, 0, 0, bn, vp(cs), vp(cs),
                                  vp(pos), 2 * (N // 3) // 64 * 64 if epi == 1 else 0, N // 2, ctypes.c_void_p(st), 0)
            assert rc == 0, rc

    def cublas():
        for i, (K, N) in enumerate(shapes):
            torch.matmul(A[K], W[i].T, out=O[i])

    for name, f in (("cublas", cublas), ("laya-store", lambda: ours(False)), ("laya-fused", lambda: ours(True))) * 2:
        for _ in range(3):
            f()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n, t0 = 0, time.time()
        e0.record()
        while time.time() - t0 < seconds:
            for _ in range(10):
                f()
            n += 10
            torch.cuda.synchronize()
        e1.record()
        e1.synchronize()
        ms = e0.elapsed_time(e1) / n
        print("%-10s M=%d: %.3f ms per set of four, %.1f TFLOP/s sustained" % (name, M, ms, flops / (ms / 1e3) / 1e12),
              flush=True)


def main():
    import torch
    from layamd_b200 import load_lib
    ap = argparse.ArgumentParser()
    ap.add_argument("--m", default="512,4096,32768,131072")
    ap.add_argument("--kn", default="1024x3072,1024x1024,1024x5248,2624x1024")
    ap.add_argument("--epi", default="store", choices=sorted(EPI))
    ap.add_argument("--modes", default="bf16,parity")
    ap.add_argument("--tile", default="auto", choices=["auto"] + sorted(TILES))
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--no-check", action="store_true")
    ap.add_argument("--no-cublas", action="store_true")
    ap.add_argument("--json", action="store_true")
    ap.add_argument("--sustained", type=float, default=0.0,
                    help="seconds: instead of the sweep, the C2 pass's four GEMMs back to back at the power cap, "
                         "cuBLAS vs this library (plain store and fused epilogues)")
    a = ap.parse_args()
    L = load_lib()
    if a.sustained > 0:
        return sustained(L, a.sustained)
    dev = torch.device("cuda:0")
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    sus, burst = peaks()
    st = torch.cuda.current_stream().cuda_stream
    rows = []
    for kn in a.kn.split(","):
        K, N = (int(x) for x in kn.split("x"))
        for M in (int(x) for x in a.m.split(",")):
            g = torch.Generator(device=dev).manual_seed(5)
            A32 = torch.randn(M, K, device=dev, generator=g)
            W32 = 0.02 * torch.randn(N, K, device=dev, generator=g)
            epi = EPI[a.epi]
            I = N // 2
            if epi == EPI["geglu"]:
                W32 = interleave_geglu(W32, I)
            ncols = I if epi == EPI["geglu"] else N

            pos = torch.randint(0, 512, (M,), device=dev, dtype=torch.int32, generator=g)
            cos = torch.rand(512, 32, device=dev)
            sin = torch.rand(512, 32, device=dev)
            for mode in a.modes.split(","):
                planes = 2 if mode == "parity" else 1
                if a.tile == "auto":
                    bn, splits = plan(L, M, N, K, sms, planes == 2)
                else:
                    bn, splits = TILES[a.tile], 1
                if planes == 1:
                    A = A32.bfloat16().contiguous()
                    W = W32.bfloat16().contiguous()
                else:
                    Ah = A32.bfloat16()
                    Wh = W32.bfloat16()
                    A = torch.stack([Ah, (A32 - Ah.float()).bfloat16()]).contiguous()
                    W = torch.stack([Wh, (W32 - Wh.float()).bfloat16()]).contiguous()
                out_mode = 2 if (planes == 2 or not a.no_check) else 0
                out = torch.empty((M, ncols), device=dev, dtype=torch.float32 if out_mode == 2 else torch.bfloat16)
                resid = torch.zeros((M, N), device=dev) if epi == EPI["resid"] else None

                def run(sync=0):
                    args = (ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(W.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                            ctypes.c_void_p(resid.data_ptr()) if resid is not None else None, None,
                            M, N, K, planes, epi, out_mode, 0, bn, ctypes.c_void_p(cos.data_ptr()),
                            ctypes.c_void_p(sin.data_ptr()), ctypes.c_void_p(pos.data_ptr()),
                            2 * (N // 3) // 64 * 64 if epi == EPI["rope"] else 0, I)
                    if splits > 1:  # the K loop in slices, partials summed by the reduce kernel
                        return L.laya_b200_gemm_splitk(*args, splits, ctypes.c_void_p(st), sync)
                    return L.laya_b200_gemm(*args, ctypes.c_void_p(st), sync)
                rc = run(1)
                assert rc == 0, rc
                err = None
                if not a.no_check and epi in (EPI["store"], EPI["resid"]):
                    ref = A32.double() @ W32.double().T
                    got = (resid if epi == EPI["resid"] else out).double()
                    err = float((got - ref).abs().max() / ref.abs().max())
                    del ref, got
                for _ in range(a.warmup):
                    run()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                torch.cuda.synchronize()
                e0.record()
                for _ in range(a.iters):
                    run()
                e1.record()
                torch.cuda.synchronize()
                ms = e0.elapsed_time(e1) / a.iters
                tf = 2.0 * M * N * K / (ms / 1e3) / 1e12
                row = {"M": M, "K": K, "N": N, "mode": mode, "epi": a.epi, "tile": bn, "splits": splits, "ms": ms,
                       "tflops": tf, "out": "f32" if out_mode == 2 else "bf16",
                       "frac_sustained": tf / sus, "frac_burst": tf / burst, "max_rel_err": err}
                if mode == "bf16" and not a.no_cublas:
                    Ab, Wb = A32.bfloat16(), W32.bfloat16()
                    for _ in range(a.warmup):
                        torch.matmul(Ab, Wb.T)
                    torch.cuda.synchronize()
                    e0.record()
                    for _ in range(a.iters):
                        torch.matmul(Ab, Wb.T)
                    e1.record()
                    torch.cuda.synchronize()
                    cms = e0.elapsed_time(e1) / a.iters
                    row["cublas_tflops"] = 2.0 * M * N * K / (cms / 1e3) / 1e12
                    del Ab, Wb
                rows.append(row)
                if a.json:
                    print(json.dumps(row), flush=True)
                else:
                    print("M=%6d K=%5d N=%5d %-6s tile=%d splits=%d %8.3f ms %7.1f TF/s (%.2f sust, %.2f burst) cublas=%s err=%s"
                          % (M, K, N, mode, bn, splits, ms, tf, tf / sus, tf / burst,
                             "%.1f" % row["cublas_tflops"] if "cublas_tflops" in row else "-",
                             "%.2e" % err if err is not None else "-"), flush=True)
                del A, W, out, resid
            del A32, W32
            torch.cuda.empty_cache()
    return rows


if __name__ == "__main__":
    sys.path.insert(0, ROOT)
    main()
