"""Write tests/golden/populations_digest.json: per population, the count of values and
refusals and a SHA-256 of the exact outputs (i64 little-endian, 0 for a refusal, followed
by the u32 refusal flags, the reference fixture's field order, native_gpu_probe.rs:234-240).

Run from the repository root: ``python tests/golden/gen_digest.py``.  The counts it
records are the ones the reference asserts (14,678 values and 32 refusals over the 14
synthetic populations, native_gpu_probe.rs:373); the digests pin the full tables so a
later change of the oracle or of the generator cannot pass silently.
"""
import hashlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from oracle import oracle  # noqa: E402
import populations as pop  # noqa: E402


def digest(values):
    v = np.array([0 if x is None else x for x in values], dtype="<i8")
    f = np.array([1 if x is None else 0 for x in values], dtype="<u4")
    return hashlib.sha256(v.tobytes() + f.tobytes()).hexdigest()


def main():
    out = {"synthetic": [], "real_quantizer": []}
    for key, cases in (("synthetic", pop.populations()),
                       ("real_quantizer", pop.real_quantizer_populations(oracle.quant_act))):
        for c in cases:
            vals = pop.exact_outputs(c, oracle.exact_dot_q8_0)
            out[key].append(dict(id=c["id"], rows=c["rows"], tokens=c["tokens"],
                                 blocks=c["blocks"],
                                 some=sum(v is not None for v in vals),
                                 refusal=sum(v is None for v in vals),
                                 sha256=digest(vals)))
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "populations_digest.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
    print(path)


if __name__ == "__main__":
    main()
