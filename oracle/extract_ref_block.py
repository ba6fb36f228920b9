"""Slice the reference's own sampling block into oracle/_ref/ (test infrastructure).

The reference keeps its sampler inline in minxfmr_generate
(src/api/minxfmr.cpp:2091-2171), so it cannot be linked on its own. This script
copies exactly that block -- from the line `int k_use = top_k;` up to, not
including, `std::string raw_tok = tokenizer_id_to_token(next);` -- out of the
reference tree into oracle/_ref/sampler_block.inc, and the pre-sampler edits
before it (special-token mask and penalties, src/api/minxfmr.cpp:2047-2089:
from the comment line that opens them up to `int k_use = top_k;`) into
oracle/_ref/edits_block.inc. ref_harness.cpp #includes them inside functions
that declare the same local variables. The slices stay in oracle/_ref/
(git-ignored); nothing from the reference is committed.

Usage: python oracle/extract_ref_block.py <reference_root> <out_dir>
Exit status 2 when the reference is absent or the anchors are not found.
"""
import hashlib
import os
import sys

START = "int k_use = top_k;"
EDITS_START = "// Suppress non-EOS special/control tokens to avoid template leakage and"
END = "std::string raw_tok = tokenizer_id_to_token(next);"
REL = os.path.join("src", "api", "minxfmr.cpp")


def main(argv):
    ref_root = argv[1] if len(argv) > 1 else "/root/reference"
    out_dir = argv[2] if len(argv) > 2 else os.path.join(os.path.dirname(__file__), "_ref")
    src = os.path.join(ref_root, REL)
    if not os.path.isfile(src):
        print(f"reference source not found: {src}", file=sys.stderr)
        return 2
    lines = open(src, encoding="utf-8", errors="replace").read().split("\n")
    starts = [i for i, l in enumerate(lines) if l.strip() == START]
    ends = [i for i, l in enumerate(lines) if l.strip() == END]
    if len(starts) != 1 or len(ends) != 1 or ends[0] <= starts[0]:
        print(f"anchors not found exactly once in {src}", file=sys.stderr)
        return 2
    block = lines[starts[0]:ends[0]]
    os.makedirs(out_dir, exist_ok=True)
    body = "\n".join(block) + "\n"
    digest = hashlib.sha256(body.encode()).hexdigest()[:16]
    with open(os.path.join(out_dir, "sampler_block.inc"), "w") as f:
        f.write(f"// sliced from {REL}:{starts[0] + 1}-{ends[0]} sha256:{digest}\n")
        f.write(body)
    print(f"{REL}:{starts[0] + 1}-{ends[0]} ({len(block)} lines) sha256:{digest}")
    e0 = [i for i, l in enumerate(lines) if l.strip() == EDITS_START]
    if len(e0) != 1 or e0[0] >= starts[0]:
        print(f"edit-block anchor not found exactly once in {src}", file=sys.stderr)
        return 2
    edits = lines[e0[0]:starts[0]]
    body = "\n".join(edits) + "\n"
    digest = hashlib.sha256(body.encode()).hexdigest()[:16]
    with open(os.path.join(out_dir, "edits_block.inc"), "w") as f:
        f.write(f"// sliced from {REL}:{e0[0] + 1}-{starts[0]} sha256:{digest}\n")
        f.write(body)
    print(f"{REL}:{e0[0] + 1}-{starts[0]} ({len(edits)} lines) sha256:{digest}")
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
