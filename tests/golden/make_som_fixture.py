"""Copies the reference's tiny model directory headers (rootfs/models/tiny/manifest.som and
index.som, 2 KB together) into tests/golden/som_tiny/, with the shard file names and sizes
of that model, so the .som reader is checked against files the reference itself wrote.
The shard files there are headerless raw tensors (an older layout that the reference's
loader, crates/soso-llm-core/src/source.rs:127, rejects as well), so they are not copied."""
import json
import os
import shutil
import sys

if len(sys.argv) != 2:
    raise SystemExit("usage: make_som_fixture.py <reference checkout>/rootfs/models/tiny")
SRC = sys.argv[1]
DST = os.path.join(os.path.dirname(os.path.abspath(__file__)), "som_tiny")

os.makedirs(DST, exist_ok=True)
for f in ("manifest.som", "index.som"):
    shutil.copyfile(os.path.join(SRC, f), os.path.join(DST, f))
shards = {f: os.path.getsize(os.path.join(SRC, "shards", f)) for f in sorted(os.listdir(os.path.join(SRC, "shards")))}
with open(os.path.join(DST, "shards.json"), "w") as fh:
    json.dump(shards, fh, indent=0, sort_keys=True)
print(f"wrote {DST}: 2 headers, {len(shards)} shard sizes")
