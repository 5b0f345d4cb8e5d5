"""Extract the known-answer values printed in the reference README.

The reference README (README.md:27-133) runs an N=2 example with
torch.manual_seed(123) on CUDA and prints, to four decimals, the projection P
and the gradient x.grad for vanilla Sinkhorn (lines 46-66), for
MHCProjectionN4 (lines 73-93) and for the low-level functions (lines
113-133).  This script reads those printed tensors from the README text and
writes them to readme_values.json next to it.

Usage (the path of the reference checkout's README is required):
    python tests/golden/make_readme_values.py <reference checkout>/README.md
"""
import json
import os
import re
import sys


def tensors_after(lines, start, count=32):
    """Parse the '# tensor([[[...' comment block that follows line `start`
    (its two 4x4 matrices are separated by an empty line)."""
    vals = []
    for line in lines[start:]:
        if line.strip() and not line.startswith("#"):
            break
        vals += [float(v) for v in re.findall(r"-?\d+\.\d+", line)]
        if len(vals) >= count:
            break
    return vals


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: make_readme_values.py <reference checkout>/README.md")
    src = sys.argv[1]
    lines = open(src).read().splitlines()
    prints = [(i, ln.strip()) for i, ln in enumerate(lines) if ln.startswith("print(")]
    names = ["P_vanilla", "dx_vanilla", "P_module", "dx_module", "P_lowlevel", "D_lowlevel"]
    assert len(prints) == len(names), prints
    out = {"source": "README.md of the reference, printed to 4 decimals",
           "print_lines": [i + 1 for i, _ in prints]}
    for name, (i, _) in zip(names, prints):
        v = tensors_after(lines, i + 1)
        assert len(v) == 32, (name, len(v))
        out[name] = v
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "readme_values.json")
    with open(dst, "w") as f:
        json.dump(out, f, indent=1)
    print("wrote", dst)


if __name__ == "__main__":
    main()
