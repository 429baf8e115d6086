"""Golden digests of the reference's MH1 checkpoint conversion (tests/golden/checkpoint_ref.json).

Writes the seeded synthetic checkpoints (lasp_b200.checkpoint, float64 and float32) and runs
the reference's own converter, built from its sources by oracle/ref/Makefile
(oracle/_ref/mace-weights-dump-ref, i.e. mace/tests/weights.cpp + mace/src/weights.cpp +
checkpoint/src/checkpoint.cpp), for every head.  Records the SHA-256 of each archive and
its record count.  Run from the repository root after building the reference tools:

    make -C oracle/ref REF=<reference tree> oracle/_ref/mace-weights-dump-ref
    python tests/golden/make_checkpoint_golden.py
"""
import hashlib
import json
import subprocess
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "lasp-pis_b200" / "python"))
import torch  # noqa: E402
from lasp_b200 import checkpoint  # noqa: E402

CASES = {"float64": (checkpoint.SEED, torch.float64), "float32": (7, torch.float32)}
TOOL = ROOT / "oracle" / "_ref" / "mace-weights-dump-ref"


def main():
    out = {"tool": "reference mace_weights_dump", "cases": {}}
    with tempfile.TemporaryDirectory() as tmp:
        for name, (seed, dtype) in CASES.items():
            model = Path(tmp) / f"mh1_{name}.model"
            checkpoint.write_checkpoint(model, seed, dtype)
            heads = {}
            for head in checkpoint.HEADS:
                pwm = Path(tmp) / "ref.pwm"
                subprocess.run([str(TOOL), str(model), str(pwm), head], check=True)
                data = pwm.read_bytes()
                heads[head] = {"sha256": hashlib.sha256(data).hexdigest(), "bytes": len(data),
                               "records": int.from_bytes(data[8:12], "little")}
            out["cases"][name] = {"seed": seed, "dtype": name, "heads": heads}
    (Path(__file__).with_name("checkpoint_ref.json")).write_text(json.dumps(out, indent=1) + "\n")


if __name__ == "__main__":
    main()
