"""Copies the small tensors of the reference's exported model (docs/model of alpha-fly, written by its
scripts/export_web.py from a trained checkpoint) into tests/golden/web/: the manifest and the tensors of at
most 100 KB.  The large blobs (synapse values and columns, encoder, policy matrix) are not copied; three of
them are missing from the reference as well (its docs/model/.MISSING_LARGE_BLOBS).

    python tests/golden/make_web_golden.py /path/to/alpha-fly/docs/model
"""
import json
import shutil
import sys
from pathlib import Path

src = Path(sys.argv[1])
dst = Path(__file__).resolve().parent / "web"
(dst / "weights").mkdir(parents=True, exist_ok=True)
manifest = json.loads((src / "manifest.json").read_text())
shutil.copyfile(src / "manifest.json", dst / "manifest.json")
copied = []
for name, t in manifest["tensors"].items():
    if t["bytes"] <= 100_000 and all((src / f).exists() for f in t["files"]):
        for f in t["files"]:
            shutil.copyfile(src / f, dst / f)
        copied.append(name)
print("copied", copied)
