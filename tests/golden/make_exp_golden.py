"""Writes exp_f64_golden.json: the reference's golden bit patterns for its portable exp.

The pairs are the `EXP_GOLDEN` table of the reference's fmath unit test
(src/domain/fmath.rs:525-550 in the redukt tree), read from the mounted source as text: 24
(input bits, output bits) pairs, including the underflow, overflow, subnormal and
round-to-1 cases.  The tests pin the C oracle's exp against them and the device exp against
the oracle.

    python tests/golden/make_exp_golden.py [/path/to/redukt]
"""
import json
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref_root=None):
    """ref_root: the redukt source tree (default: $REDUKT_REF_ROOT, else `reference` beside the repo)."""
    if ref_root is None:
        sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
        from oracle.oracle import reference_root
        ref_root = reference_root()
        if ref_root is None:
            raise SystemExit("the redukt source tree was not found: set REDUKT_REF_ROOT")
    src = open(os.path.join(ref_root, "src", "domain", "fmath.rs")).read()
    body = re.search(r"const EXP_GOLDEN: \[\(f64, u64\); \d+\] = \[(.*?)\];", src, re.S).group(1)
    pairs = re.findall(r"f64::from_bits\(0x([0-9a-f]+)\), 0x([0-9a-f]+)\)", body)
    out = {"source": "src/domain/fmath.rs:525-550 (EXP_GOLDEN)",
           "pairs": [[f"0x{x}", f"0x{y}"] for x, y in pairs]}
    with open(os.path.join(HERE, "exp_f64_golden.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(f"wrote {len(pairs)} pairs")


if __name__ == "__main__":
    main(*sys.argv[1:])
