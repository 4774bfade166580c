"""Regenerate the golden fixtures in this folder from the reference checkout.

The reference (a Rust workspace) cannot be built or imported here, so its own
parity fixtures are the golden vectors.  This script copies the tensors of
those fixtures (unchanged bytes, same names, same __metadata__ plus a
`source` entry naming the reference file) into tests/golden/, so the tests
and the GPU box, which has no reference checkout, can read them.

Sources (paths inside the reference project):
  crates/ltx-weights/tests/fixtures/*.safetensors   (FP8 dequant, LoRA merge,
      transformer key map, IC-LoRA layout; generator tools/parity/ltx-weights.py)
  crates/ltx-dit/tests/fixtures/dit_parity*.safetensors  (tiny DiT forward;
      generator tools/parity/ltx-dit.py, upstream LTX-2 commit 9ec55f9)

Usage:  python tests/golden/make_golden.py <reference_root>
"""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle.weight_store import read_safetensors, write_safetensors  # noqa: E402

FIXTURES = [
    "crates/ltx-weights/tests/fixtures/fp8_e4m3fn_parity.safetensors",
    "crates/ltx-weights/tests/fixtures/fp8_e4m3fn_expected.safetensors",
    "crates/ltx-weights/tests/fixtures/lora_parity_base.safetensors",
    "crates/ltx-weights/tests/fixtures/lora_parity_lora.safetensors",
    "crates/ltx-weights/tests/fixtures/lora_parity_expected.safetensors",
    "crates/ltx-weights/tests/fixtures/transformer_keymap_fixture.safetensors",
    "crates/ltx-weights/tests/fixtures/transformer_keymap_expected.safetensors",
    "crates/ltx-weights/tests/fixtures/iclora_layout.safetensors",
    "crates/ltx-dit/tests/fixtures/dit_parity.safetensors",
    "crates/ltx-dit/tests/fixtures/dit_parity_gated_adaln.safetensors",
]


def main(ref_root):
    for rel in FIXTURES:
        meta, tensors = read_safetensors(os.path.join(ref_root, rel))
        meta = dict(meta)
        meta["source"] = rel
        out = os.path.join(HERE, os.path.basename(rel))
        write_safetensors(out, tensors, meta)
        print("wrote", out, len(tensors), "tensors")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference_root>  (the ltx-rust checkout)")
    main(sys.argv[1])
