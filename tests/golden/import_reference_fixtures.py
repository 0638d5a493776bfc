"""Copy the reference's weight-free golden vectors into tests/golden/ref/.

The RCuteTTS crate ships .npy fixtures that need no checkpoint: the M1 op
fixtures (tests/m1_ops.rs:33-110, made by scripts/dump_m1_fixtures.py from
the torch audio_vae.py modules) and the base sway grid (tests/dit_base.rs:39-49).
They are data produced by the reference's own torch code; this script copies
them verbatim so the CPU parity tests can pin the oracle without the
reference tree being present.  It also records the shipped checkpoints'
tensor lists from the crate's manifests (ref/manifests.json) for the
checkpoint-loading tests.

Usage: python tests/golden/import_reference_fixtures.py [REFERENCE_ROOT]
"""
import json
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


# The shipped checkpoints' tensor lists (name -> shape, dtype), as recorded by
# the crate's manifests (rust-codec/*_manifest.json): the loader interface the
# device loaders must accept.
MANIFESTS = {"lm": "qwen_manifest.json", "dit": "dit_manifest.json", "locenc": "locenc_manifest.json",
             "vae": "weights_manifest.json"}


def import_manifests(root: str, dst: str) -> None:
    out = {}
    for key, fn in MANIFESTS.items():
        with open(os.path.join(root, "rust-codec", fn)) as f:
            m = json.load(f)
        if key == "vae":
            m = m["decoder"]
        out[key] = {name: [list(v["shape"]), v["dtype"].replace("torch.", "")] for name, v in sorted(m.items())}
    with open(os.path.join(dst, "manifests.json"), "w") as f:
        json.dump(out, f, indent=0, sort_keys=True)
    print("manifests:", {k: len(v) for k, v in out.items()})


def main(root: str) -> None:
    src = os.path.join(root, "rust-codec", "testdata")
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "ref")
    os.makedirs(dst, exist_ok=True)
    for n in NAMES:
        shutil.copyfile(os.path.join(src, n + ".npy"), os.path.join(dst, n + ".npy"))
    print(f"copied {len(NAMES)} fixtures to {dst}")
    import_manifests(root, dst)


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("RCUTETTS_REFERENCE", "")
    if not root:
        sys.exit("usage: import_reference_fixtures.py <RCuteTTS checkout> (or set RCUTETTS_REFERENCE)")
    main(root)
