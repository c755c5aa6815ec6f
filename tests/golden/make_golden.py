#!/usr/bin/env python3
"""Regenerates the golden vectors under tests/golden/ from ctorch itself.

  ctorch_parity_fixtures.npz  ctorch's own parity fixtures (tests/parity/fixtures/*.npy in the
                              ctorch tree, produced there by scripts/gen_parity.py), repacked
                              into one file so tests can read them without the ctorch tree.
  ctorch_ref_cases.npz        the seeded cases of catalog.py, run through ctorch's CPU backend
                              (oracle/_ref/libctorch_ref.so, ctorch's sources compiled in place)
                              via its public front-doors and view ops. Stores inputs, outputs or
                              the ctorch error code.

Usage: python tests/golden/make_golden.py [--ctorch-dir /root/reference]
(needs `make -C oracle ref` first).
"""
from __future__ import annotations

import argparse
import glob
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.abspath(os.path.join(HERE, "..", ".."))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

from catalog import apply_ref, cases  # noqa: E402
from oracle.oracle import Ref, RefError  # noqa: E402


def run_ref(ref: Ref, case):
    ins = [apply_ref(ref.tensor(base), recipe) for base, recipe in case.inputs]
    kw = case.kw
    if case.kind == "binary":
        return [ref.binary(case.op, ins[0], ins[1]).numpy()]
    if case.kind == "inplace":
        ref.binary_inplace(case.op, ins[0], ins[1])
        return [ins[0].numpy()]
    if case.kind == "unary":
        return [ref.unary(case.op, ins[0]).numpy()]
    if case.kind == "reduce":
        return [ref.reduce(case.op, ins[0], kw["dims"], kw["keepdim"]).numpy()]
    if case.kind == "reduce_idx":
        v, i = ref.reduce_idx(case.op, ins[0], kw["dim"], kw["keepdim"])
        return [v.numpy(), i.numpy()]
    if case.kind == "arg":
        return [ref.arg(case.op, ins[0], kw["dim"], kw["keepdim"]).numpy()]
    if case.kind == "index_select":
        return [ref.index_select(ins[0], kw["dim"], ins[1]).numpy()]
    raise ValueError(case.kind)


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--ctorch-dir", default="/root/reference")
    args = ap.parse_args()

    fix_dir = os.path.join(args.ctorch_dir, "tests", "parity", "fixtures")
    fixtures = {os.path.basename(p)[:-4]: np.load(p) for p in sorted(glob.glob(os.path.join(fix_dir, "*.npy")))}
    np.savez_compressed(os.path.join(HERE, "ctorch_parity_fixtures.npz"), **fixtures)
    print(f"repacked {len(fixtures)} ctorch parity fixtures")

    ref = Ref()
    store = {}
    names = []
    for c in cases():
        names.append(c.name)
        store[f"{c.name}/meta"] = np.array(c.meta())
        for k, (base, _) in enumerate(c.inputs):
            store[f"{c.name}/in{k}"] = base
        try:
            outs = run_ref(ref, c)
            store[f"{c.name}/status"] = np.array(0)
            for k, o in enumerate(outs):
                store[f"{c.name}/out{k}"] = o
        except RefError as e:
            store[f"{c.name}/status"] = np.array(e.code)
    store["__names__"] = np.array(names)
    np.savez_compressed(os.path.join(HERE, "ctorch_ref_cases.npz"), **store)
    print(f"wrote {len(names)} ctorch-run cases")


if __name__ == "__main__":
    main()
