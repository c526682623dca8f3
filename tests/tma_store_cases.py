"""GEMM cases whose outputs the tensor-map (TMA) epilogue and the register-store epilogue
must write identically: ragged pair tiles with bias + ReLU, batched pair tiles with a row
bias, one-CTA tiles, config 3's broadcast bmm, and a C window inside a larger buffer
whose surroundings must stay untouched. Run directly, it writes every output (and the
guard-band buffer) to the .npz named on the command line; the process reads
MT_TMA_EPILOGUE once, at the first GEMM, so each setting needs its own process."""
import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from minitensor_b200 import engine, inputs  # noqa: E402


def _dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def run_cases():
    """{name: output array} and {name: path} for every case, in both precisions."""
    out, paths = {}, {}
    for mode in ("tf32", "tf32x3"):
        # CTA-pair tiles, ragged edges (K = 301 inside rows of 304 so that TMA can load
        # A; N = 2356 keeps C's rows 16-byte aligned, off the 32-column blocks), column
        # bias + ReLU.
        M, N, K = 2381, 2356, 301
        A = _dev(inputs.uniform((M, 304), -1, 1, 191))[:, :K]
        B = _dev(inputs.uniform((K, N), -1, 1, 192))
        bn = _dev(inputs.uniform((N,), -1, 1, 193))
        C = torch.empty(M, N, device="cuda")
        engine.gemm(A, B, C, bias=bn, epi=engine.EPI_BIAS_COL | engine.EPI_RELU, mode=mode)
        out[f"pair_{mode}"], paths[f"pair_{mode}"] = C.cpu().numpy(), engine.last_path()
        # Batched pair tiles, row bias.
        Bt, M, N, K = 3, 1290, 1100, 200
        A = _dev(inputs.uniform((Bt, M, K), -1, 1, 194))
        B = _dev(inputs.uniform((Bt, K, N), -1, 1, 195))
        bm = _dev(inputs.uniform((M,), -1, 1, 196))
        C = torch.empty(Bt, M, N, device="cuda")
        engine.gemm(A, B, C, bias=bm, epi=engine.EPI_BIAS_ROW, mode=mode)
        out[f"batched_{mode}"], paths[f"batched_{mode}"] = C.cpu().numpy(), engine.last_path()
        # One-CTA tiles (too few 256 x 256 tiles for pairs), M and N off the 32-row blocks.
        M, N, K = 700, 612, 96
        A = _dev(inputs.uniform((M, K), -1, 1, 197))
        B = _dev(inputs.uniform((K, N), -1, 1, 198))
        C = torch.empty(M, N, device="cuda")
        engine.gemm(A, B, C, mode=mode)
        out[f"single_{mode}"], paths[f"single_{mode}"] = C.cpu().numpy(), engine.last_path()
        # Config 3: 64 x [512x64].[64x512], B broadcast over the batch.
        A_h, B0_h = inputs.config3()
        B0 = _dev(B0_h)
        C = torch.empty(64, 512, 512, device="cuda")
        engine.gemm(_dev(A_h), B0.expand(64, 64, 512), C, mode=mode)
        out[f"config3_{mode}"], paths[f"config3_{mode}"] = C.cpu().numpy(), engine.last_path()
        # C as a window of a larger buffer (row stride 1044, 4-column offset).
        M, N, K = 1030, 1000, 64
        A = _dev(inputs.uniform((M, K), -1, 1, 199))
        B = _dev(inputs.uniform((K, N), -1, 1, 200))
        big = torch.full((M + 16, N + 44), 12345.0, device="cuda")
        engine.gemm(A, B, big[8:8 + M, 4:4 + N], mode=mode)
        out[f"window_{mode}"], paths[f"window_{mode}"] = big.cpu().numpy(), engine.last_path()
    torch.cuda.synchronize()
    return out, paths


if __name__ == "__main__":
    torch.cuda.set_device(0)
    engine.lib()
    o, p = run_cases()
    np.savez(sys.argv[1], **o, **{"path_" + k: np.array(v) for k, v in p.items()})
