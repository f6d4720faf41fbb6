"""Regenerates tests/golden/oracle_vectors.json from the C oracle.

The vectors freeze the oracle's key chain (step_key -> candidate_key ->
group_key -> factor keys), raw bits and float32 normals for a few seeds, so a
change to the oracle or to the device PRNG shows up as a fixture mismatch.
Run: python tests/golden/make_golden.py
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import ref  # noqa: E402


def main():
    out = {"step_keys": [], "chains": [], "streams": []}
    for seed, run, gen, ver in [(0, "bench", 0, 1), (42, "test", 0, 1), (42, "run", 3, 1), (7, "x" * 40, 123456, 9)]:
        out["step_keys"].append({"seed": seed, "run_id": run, "generation": gen, "version": ver,
                                 "key": [int(v) for v in ref.step_key(seed, run, gen, ver)]})
    base = ref.step_key(42, "test", 0, 1)
    ids = list(range(8))
    cks = ref.candidate_keys(base, ids)
    for g in range(3):
        gks = ref.group_keys(cks, g)
        ka = np.stack([ref.split(k)[0] for k in gks])
        kb = np.stack([ref.split(k)[1] for k in gks])
        out["chains"].append({"base": [int(v) for v in base], "ids": ids, "group": g,
                              "candidate_keys": cks.tolist(), "group_keys": gks.tolist(),
                              "factor_a_keys": ka.tolist(), "factor_b_keys": kb.tolist()})
    for k in ([0, 0], [0, 42], [0x12345678, 0x9ABCDEF0]):
        kk = np.array(k, np.uint32)
        bits = ref.random_bits(kk, 64)
        nrm = ref.normal(kk, (64,))
        out["streams"].append({"key": k, "bits": bits.tolist(),
                               "normal_f32_bits": nrm.view(np.uint32).tolist()})
    with open(os.path.join(HERE, "oracle_vectors.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
