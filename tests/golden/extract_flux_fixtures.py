"""Extract the golden vectors the FLUX tests pin against from the reference's
own test fixtures into one committed file.

Run from the repository root, with the reference's fixture directory (its
inst/tinytest/fixtures) as the argument:

    python tests/golden/extract_flux_fixtures.py <reference>/inst/tinytest/fixtures

It reads `flux_model.safetensors` (the tiny FLUX transformer: its weights, its
inputs and the output the reference's generator recorded) and
`rope_flux.safetensors` (rotary tables, rotary application, latent packing),
and writes every tensor unchanged to `flux_reference_fixtures.safetensors`
beside this script, each key prefixed with its source file's stem.
"""
import os
import sys

from safetensors.torch import load_file, save_file

SOURCES = ("flux_model", "rope_flux")
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "flux_reference_fixtures.safetensors")


def main(src_dir: str) -> None:
    out = {}
    for stem in SOURCES:
        for k, v in load_file(os.path.join(src_dir, stem + ".safetensors")).items():
            out[f"{stem}/{k}"] = v.contiguous()
    save_file(out, OUT)
    print(f"wrote {len(out)} tensors to {OUT}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])
