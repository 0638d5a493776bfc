"""Copy the reference's weight-free golden vectors into tests/golden/ref/.

The RCuteTTS crate ships .npy fixtures that need no checkpoint: the M1 op
fixtures (tests/m1_ops.rs:33-110, made by scripts/dump_m1_fixtures.py from
the torch audio_vae.py modules) and the base sway grid (tests/dit_base.rs:39-49).
They are data produced by the reference's own torch code; this script copies
them verbatim so the CPU parity tests can pin the oracle without the
reference tree being present.

Usage: python tests/golden/import_reference_fixtures.py [REFERENCE_ROOT]
"""
import os
import shutil
import sys

NAMES = [
    "m1_conv_d3_in", "m1_conv_d3_w", "m1_conv_d3_b", "m1_conv_d3_out",
    "m1_conv_dw9_in", "m1_conv_dw9_w", "m1_conv_dw9_b", "m1_conv_dw9_out",
    "m1_trans_s16_in", "m1_trans_s16_w", "m1_trans_s16_b", "m1_trans_s16_out",
    "m1_trans_s3_in", "m1_trans_s3_w", "m1_trans_s3_b", "m1_trans_s3_out",
    "m1_resunit_d3_in", "m1_resunit_d3_w0", "m1_resunit_d3_b0", "m1_resunit_d3_w1",
    "m1_resunit_d3_b1", "m1_resunit_d3_out",
    "m1_snake_in", "m1_snake_alpha", "m1_snake_out",
    "base_sway",
]


def main(root: str) -> None:
    src = os.path.join(root, "rust-codec", "testdata")
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ref")
    os.makedirs(dst, exist_ok=True)
    for n in NAMES:
        shutil.copyfile(os.path.join(src, n + ".npy"), os.path.join(dst, n + ".npy"))
    print(f"copied {len(NAMES)} fixtures to {dst}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
