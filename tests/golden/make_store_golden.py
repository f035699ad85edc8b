"""Generate the expert-store fixture that pins moeb200.store to the reference's store format.

Run in the build container, where the reference (moelab) is importable from its read-only checkout
and transformers is installed:

    MOELAB_ROOT=<path to the moelab checkout> python tests/golden/make_store_golden.py

A tiny random OLMoE checkpoint (moelab.testing: 2 MoE layers of 4 experts, H=64, I=32) is
converted by the reference's own moelab.store.build_store into tests/golden/store_tiny/ (fp16 and
int4 records, absmax scales); store_tiny_meta.json records the SHA-256 of every record as the
reference's ExpertStore.read returns it.
"""

from __future__ import annotations

import hashlib
import json
import os
import shutil
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, os.environ.get("MOELAB_ROOT", "/root/reference"))

from moelab.store import ExpertStore, build_store  # noqa: E402
from moelab.testing import make_model_dir, tiny_olmoe_config  # noqa: E402

out = HERE / "store_tiny"
if out.exists():
    shutil.rmtree(out)
with tempfile.TemporaryDirectory() as tmp:
    model = make_model_dir(Path(tmp) / "model", tiny_olmoe_config(num_hidden_layers=2, num_experts=4), seed=3)
    build_store(model, out, precisions=("fp16", "int4"), int4_scale="absmax", device="cpu", log=lambda *a: None)
for extra in ("progress.json",):
    if (out / extra).exists():
        (out / extra).unlink()
# the manifest names the converted checkpoint's (temporary) directory; keep a stable description
man = json.loads((out / "manifest.json").read_text(encoding="utf-8"))
man["source"] = "tiny random OLMoE (moelab.testing.tiny_olmoe_config, 2 layers, 4 experts, seed 3)"
(out / "manifest.json").write_text(json.dumps(man, indent=1), encoding="utf-8")
st = ExpertStore(out)
meta = {"num_experts": st.num_experts, "hidden": st.hidden, "inter": st.inter, "layers": st.layers,
        "precisions": st.precisions, "record_sha256": {}}
for li in range(len(st.layers)):
    for e in range(st.num_experts):
        for p in st.precisions:
            blob = st.read(li, e, p)
            meta["record_sha256"][f"{li}:{e}:{p}"] = hashlib.sha256(blob.numpy().tobytes()).hexdigest()
st.close()
(HERE / "store_tiny_meta.json").write_text(json.dumps(meta, indent=1) + "\n")
print("wrote", out, sum(f.stat().st_size for f in out.iterdir()), "bytes")
