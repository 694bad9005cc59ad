"""Stage the unmodified reference for the GPU reference arm and the drop-in tests
(TEST AND BASELINE INFRASTRUCTURE ONLY; nothing staged is committed).

  * baseline/_ref/            the reference package spikeDE_dis, installed with pip from a
                              copy of the checkout (the checkout is read-only; its
                              requirements -- cupy, timm, spikingjelly, h5py -- are not
                              installable offline, so --no-deps);
  * baseline/_ref/examples/   the example modules the network tests import unmodified:
                              cnn128/{cnn128_aligned,aligned_glmulti}.py and
                              spikformer_har_lip/{model,aligned_glmulti}.py.

Both folders are git-ignored and travel with the working tree.

Usage: python oracle/stage_ref.py [--reference PATH] [--force]
"""
import argparse
import os
import shutil
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
TARGET = os.path.join(REPO, "baseline", "_ref")
EXAMPLES = {"cnn128": ("cnn128_aligned.py", "aligned_glmulti.py"),
            "spikformer_har_lip": ("model.py", "aligned_glmulti.py")}


def stage(reference, force=False):
    if not os.path.isdir(os.path.join(reference, "spikeDE_dis")):
        print(f"stage_ref: no reference checkout at {reference}; skipped")
        return None
    if force or not os.path.isdir(os.path.join(TARGET, "spikeDE_dis")):
        with tempfile.TemporaryDirectory() as tmp:
            src = os.path.join(tmp, "reference")
            shutil.copytree(reference, src, ignore=shutil.ignore_patterns(".git"))
            subprocess.check_call([sys.executable, "-m", "pip", "install", "--quiet",
                                   "--no-index", "--no-build-isolation", "--no-deps",
                                   "--find-links", "/opt/wheelhouse", "--upgrade",
                                   "--target", TARGET, src])
    for name, files in EXAMPLES.items():
        dst = os.path.join(TARGET, "examples", name)
        os.makedirs(dst, exist_ok=True)
        for fn in files:
            shutil.copyfile(os.path.join(reference, "examples", name, fn), os.path.join(dst, fn))
    print(f"stage_ref: reference staged in {TARGET}")
    return TARGET


if __name__ == "__main__":
    sys.path.insert(0, HERE)
    from build_ref import reference_path
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    stage(reference_path(args.reference), args.force)
