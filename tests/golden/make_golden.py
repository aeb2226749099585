"""Regenerates the golden fixtures in this directory from the reference itself.

Run where the reference tree is present, after building the reference-compiled oracle
libraries (make -C oracle REF=<reference tree>):

    python tests/golden/make_golden.py --ref <reference tree>

(--ref defaults to the environment variable CKL_REFERENCE.)

Fixtures written (all small):
  moe_decode_counts.json  per-expert routed counts published by the reference
                          (results/moe_decode_counts.txt), with the shapes they belong to
  attn_config1.npz        BASELINE config 1 -- Batch({1000,777}, 32, 8, seed 7): the
                          reference's own cpu_reference output (out, lse) plus SHA-256
                          digests of the generated q/k/v/page table
  cascade_case1.npz       make_shared_prefix_batch(64, {1,17,40}, Hq=8, Hkv=8, seed 13)
                          (01_decode_attention.cu:783): cpu_reference out/lse + digests
  known_answers.json      shared_prefix_pages of the unshared batch
                          Batch(4x1000, 32, 8, seed 3) (01_decode_attention.cu:810-815)
"""
import argparse
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import oracle as O  # noqa: E402


def digests(bt):
    d = {}
    for name in ("indptr", "indices", "last", "q", "k", "v"):
        a = getattr(bt, name)
        d[name] = hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
    return d


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("CKL_REFERENCE"),
                    help="the reference tree (default: $CKL_REFERENCE)")
    args = ap.parse_args()
    if not args.ref or not os.path.isdir(args.ref):
        sys.exit("make_golden: pass --ref <reference tree> (or set CKL_REFERENCE)")
    if O.ref01() is None or O.ref03() is None:
        sys.exit("oracle/_ref libraries missing: run make -C oracle (needs the reference tree)")

    rows = []
    with open(os.path.join(args.ref, "results", "moe_decode_counts.txt")) as f:
        for line in f:
            v = [int(x) for x in line.split()]
            rows.append({"T": v[0], "E": v[1], "d": v[2], "f": v[3], "seed": 9,
                         "k": 6 if v[1] == 64 else 2, "counts": v[4:]})
    with open(os.path.join(HERE, "moe_decode_counts.json"), "w") as f:
        json.dump({"source": "results/moe_decode_counts.txt (03_moe_wq_decode.cu:501-517)",
                   "note": "produced by an MSVC build: normal draws in MSVC pair order",
                   "rows": rows}, f, indent=1)

    bt = O.ref_batch([1000, 777], 32, 8, 7)
    out, lse = O.ref_cpu_reference(bt)
    np.savez_compressed(os.path.join(HERE, "attn_config1.npz"), out=out, lse=lse,
                        **{"sha_" + k: v for k, v in digests(bt).items()})

    bt = O.ref_shared_prefix_batch(64, [1, 17, 40], 8, 8, 13)
    out, lse = O.ref_cpu_reference(bt)
    np.savez_compressed(os.path.join(HERE, "cascade_case1.npz"), out=out, lse=lse,
                        **{"sha_" + k: v for k, v in digests(bt).items()})

    un = O.ref_batch([1000] * 4, 32, 8, 3, fill=False)
    pages = O.ref01().ref01_shared_prefix_pages(O._p(un.indptr), O._p(un.indices), un.B)
    with open(os.path.join(HERE, "known_answers.json"), "w") as f:
        json.dump({"unshared_batch_4x1000_seed3_shared_pages": pages}, f, indent=1)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
