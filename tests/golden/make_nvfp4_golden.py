"""Generate tests/golden/nvfp4_intrinsics.npz: results of the CUDA header intrinsics the
reference's NVFP4 quantisers call, evaluated on the host (no GPU needed).

    python tests/golden/make_nvfp4_golden.py      # needs nvcc

Compiles nvfp4_intrinsics_host.cu (beside this file) with nvcc, runs it and stores
  e4m3_decode[256]          every E4M3 code as float
  e4m3_in_bits / e4m3_code  float bit patterns and their E4M3 code (round-nearest, SATFINITE)
  fp4_a / fp4_b / fp4_byte  float pairs and the packed e2m1x2 byte (round-nearest)
"""
import os
import struct
import subprocess
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main():
    with tempfile.TemporaryDirectory() as d:
        exe, tab = os.path.join(d, "gen"), os.path.join(d, "table.bin")
        subprocess.check_call(["nvcc", "-O1", "-o", exe, os.path.join(HERE, "nvfp4_intrinsics_host.cu")])
        subprocess.check_call([exe, tab])
        raw = open(tab, "rb").read()
    off = 0
    dec = np.frombuffer(raw, np.float32, 256, off).copy(); off += 1024
    (n,) = struct.unpack_from("<I", raw, off); off += 4
    rec = np.frombuffer(raw, np.dtype([("bits", "<u4"), ("code", "u1")]), n, off); off += 5 * n
    (m,) = struct.unpack_from("<I", raw, off); off += 4
    rec2 = np.frombuffer(raw, np.dtype([("a", "<f4"), ("b", "<f4"), ("p", "u1")]), m, off)
    out = os.path.join(HERE, "nvfp4_intrinsics.npz")
    np.savez_compressed(out, e4m3_decode=dec, e4m3_in_bits=rec["bits"].copy(), e4m3_code=rec["code"].copy(),
                        fp4_a=rec2["a"].copy(), fp4_b=rec2["b"].copy(), fp4_byte=rec2["p"].copy())
    print("wrote", out, os.path.getsize(out), "bytes;", n, "e4m3 samples,", m, "fp4 pairs")


if __name__ == "__main__":
    main()
