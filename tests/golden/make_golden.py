"""Generate the golden fixtures in this directory from the reference's own gates.

Run where the reference checkout is present (ROCKET_REF, else a directory
named "reference" beside this repository).  For each gate below this script:
  1. builds oracle/_ref/pin_<gate> (the reference's test program compiled
     unchanged, linked against oracle/ref_stub.c + oracle/oracle.c),
  2. runs it with ORC_DUMP set, so every matmul call the gate makes dumps its
     inputs and the oracle's output,
  3. requires the gate's own verdict to be PASS (its host loop, its seeded
     glibc rand() inputs, its tolerance), and
  4. writes <name>.npz with the inputs and expected output, plus an entry in
     manifest.json recording the gate, its arguments and its PASS line.

The fixtures are what the GPU tests compare the CUDA path against on the GPU
box (where the reference tree is absent).
"""
from __future__ import annotations

import json
import os
import struct
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
ORACLE = os.path.join(REPO, "oracle")

# (fixture name, gate, argv, which dumped call to keep)
CASES = [
    ("int8_config1", "matmul_int8_tiled_rocket", ["64", "512", "256"], 0),
    ("int8_ragged", "matmul_int8_tiled_rocket", ["12", "96", "64"], 0),
    ("fp16_small", "matmul_tiled_rocket", ["32", "256", "128"], 0),
    ("fp16_m1", "matmul_tiled_rocket", ["1", "64", "48"], 0),
    ("int8_gw_g96", "matmul_int8_groupwise_rocket", ["32", "576", "64", "96"], 0),
    ("int4_gw_g128", "matmul_int4_groupwise_rocket", ["32", "512", "128", "128"], 0),
    ("int4_prepacked", "matmul_int4_prepacked_rocket", ["16", "256", "128", "1"], 0),
]

DT = {"int8": (np.int8, np.int8, np.int32), "int4": (np.int8, np.int8, np.int32),
      "fp16": (np.float16, np.float16, np.float16),
      "int8_gw": (np.int8, np.int8, np.float32), "int4_gw": (np.int8, np.int8, np.float32)}


def read_dump(path):
    with open(path, "rb") as f:
        data = f.read()
    assert data[:4] == b"RKBG"
    kind = data[4:20].split(b"\0")[0].decode()
    M, K, N, group = struct.unpack("<4i", data[20:36])
    sizes = struct.unpack("<5Q", data[36:76])
    off = 76
    arrs = []
    for s in sizes:
        arrs.append(data[off:off + s])
        off += s
    ta, tb, tc = DT[kind]
    out = {"kind": kind, "M": M, "K": K, "N": N, "group": group,
           "A": np.frombuffer(arrs[0], ta).reshape(M, K),
           "B": np.frombuffer(arrs[1], tb).reshape(N, K),
           "C": np.frombuffer(arrs[4], tc).reshape(M, N)}
    if sizes[2]:
        nG = K // group
        out["a_scale"] = np.frombuffer(arrs[2], np.float32).reshape(M, nG)
        out["b_scale"] = np.frombuffer(arrs[3], np.float32).reshape(N, nG)
    return out


def main():
    subprocess.run(["make", "-C", ORACLE, "pin"], check=True)
    manifest = {}
    for name, gate, argv, keep in CASES:
        exe = os.path.join(ORACLE, "_ref", "pin_" + gate)
        with tempfile.TemporaryDirectory() as td:
            env = dict(os.environ, ORC_DUMP=os.path.join(td, "d"))
            r = subprocess.run([exe] + argv, env=env, capture_output=True, text=True, timeout=600)
            verdicts = [l for l in r.stdout.splitlines() if "PASS" in l or "FAIL" in l]
            if r.returncode != 0 or not verdicts or any("FAIL" in v for v in verdicts):
                print(r.stdout, r.stderr)
                sys.exit(f"gate {gate} {argv} did not pass")
            dumps = sorted(os.listdir(td))
            d = read_dump(os.path.join(td, dumps[keep]))
        arrays = {k: v for k, v in d.items() if isinstance(v, np.ndarray)}
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrays)
        manifest[name] = {"gate": f"tests/{gate}.c", "argv": argv, "kind": d["kind"],
                          "M": d["M"], "K": d["K"], "N": d["N"], "group": d["group"],
                          "gate_verdict": verdicts[-1].strip()}
        print(name, manifest[name]["gate_verdict"])
    with open(os.path.join(HERE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)


if __name__ == "__main__":
    main()
