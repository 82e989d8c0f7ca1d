"""Regenerate the committed golden fixtures from the reference checkout.

Run in the build container (the reference tree is not present on GPU boxes):

    python tests/golden/make_golden.py --reference <path to the reference tree>

Writes, next to this script:

* ``fp8_cast.json``  -- the 12 quantizer cases of the reference's
  ``crates/reng-fp8/fixtures/fp8_cast.json`` (bf16 weights, scale bits, codes,
  torch's raw bytes for the saturation cases, numpy row errors), with the
  fields the tests read.  Shared-weight cases keep their ``bf16_from`` link.
* ``rope_reference.json`` -- the 10 RoPE cases of the reference's
  ``crates/reng-model/testdata/rope_reference.json`` (transformers tables at
  sampled positions, with each case's config.json).

The data are the reference's own golden vectors; this script only selects
fields, so the fixture files are byte-for-byte reproducible from it.
"""
import argparse
import json
import os

HERE = os.path.dirname(os.path.abspath(__file__))

FP8_KEYS = ("name", "format", "scaling", "exp_bias", "rows", "cols", "bf16_hex",
            "bf16_from", "scale_bits", "codes_hex", "torch_raw_hex",
            "torch_bytes_saturated", "mean_rel", "max_rel")


def fp8(ref):
    src = os.path.join(ref, "crates/reng-fp8/fixtures/fp8_cast.json")
    with open(src) as f:
        doc = json.load(f)
    out = {
        "source": "reference crates/reng-fp8/fixtures/fp8_cast.json",
        "generator": doc["generator"],
        "torch": doc["torch"],
        "numpy": doc["numpy"],
        "model": doc["model"],
        "cases": [{k: c[k] for k in FP8_KEYS if k in c} for c in doc["cases"]],
    }
    with open(os.path.join(HERE, "fp8_cast.json"), "w") as f:
        json.dump(out, f, indent=0, sort_keys=True)
        f.write("\n")
    return len(out["cases"])


def rope(ref):
    src = os.path.join(ref, "crates/reng-model/testdata/rope_reference.json")
    with open(src) as f:
        doc = json.load(f)
    cases = []
    for c in doc["cases"]:
        cases.append(dict(c))
    out = {"source": "reference crates/reng-model/testdata/rope_reference.json",
           "transformers": doc["transformers"], "torch": doc["torch"], "cases": cases}
    with open(os.path.join(HERE, "rope_reference.json"), "w") as f:
        json.dump(out, f, indent=0, sort_keys=True)
        f.write("\n")
    return len(cases)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="the reference checkout (its crates/ tree)")
    a = ap.parse_args()
    print("fp8 cases", fp8(a.reference))
    print("rope cases", rope(a.reference))


if __name__ == "__main__":
    main()
