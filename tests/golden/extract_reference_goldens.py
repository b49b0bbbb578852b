"""Copies the det (not fp32) commitments of the reference's golden file.

Source: casettek/raster-inference testdata/det_commitment_goldens.json
(written by src/runtime/det_goldens.rs).  Run where the reference checkout
is available; the output det_commitment_goldens.json is committed so that
tests never read the reference at run time.

    python tests/golden/extract_reference_goldens.py /path/to/raster-inference
"""
import json
import os
import sys

if len(sys.argv) < 2:
    sys.exit("usage: extract_reference_goldens.py <raster-inference checkout>")
src = os.path.join(sys.argv[1], "testdata/det_commitment_goldens.json")
with open(src) as f:
    g = json.load(f)
out = {name: {"det": fx["det"]} for name, fx in g.items()}
dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "det_commitment_goldens.json")
with open(dst, "w") as f:
    json.dump(out, f, indent=1, sort_keys=True)
print("wrote", dst)
