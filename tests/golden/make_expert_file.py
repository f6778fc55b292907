"""Golden record of the reference's expert-file format (tests/golden/expert_file.json).

Runs, from a reference checkout given as argv[1], the reference's own converter step
(scripts/convert-mimo-v26-mlx.py:92-131 `convert_expert_layer` + `write_safetensors`) on seeded
expert bytes with the projection shapes shrunk (PROJ is a module table; the layout logic is
untouched), then the reference's own reader (engine/mimo_stream/store.py `ExpertStore` + `IOPool`,
fcntl's macOS-only cache hints stubbed out) on the file it wrote.  Records the file's size and SHA-256,
every tensor's (base, stride) as ExpertStore computes them, and the SHA-256 of each slice of one expert
as IOPool reads it.  The file itself is not committed (832 KiB); the tests rebuild it with the
package's writer from the same bytes and compare.

    python tests/golden/make_expert_file.py <reference checkout>
"""
from __future__ import annotations

import hashlib
import importlib.util
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LAYER, N_EXP, PROBE_EXPERT = 5, 4, 2
# (out, in) per projection: small, and still every stacked tensor a multiple of 16 KiB
SHAPES = {"gate_proj": (128, 1024), "up_proj": (128, 1024), "down_proj": (1024, 128)}


def fixture_bytes(proj: str, kind: str, e: int, n: int) -> bytes:
    """Seeded bytes of expert e's `kind` ("weight" or "weight_scale") of `proj` (splitmix64 stream)."""
    tag = list(SHAPES).index(proj) * 2 + (kind == "weight_scale")
    j = np.arange(1, n // 8 + 2, dtype=np.uint64)
    z = (j + np.uint64(1000 * tag + e)) * np.uint64(0x9E3779B97F4A7C15)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z = z ^ (z >> np.uint64(31))
    return z.view(np.uint8)[:n].tobytes()


def fixture_arrays():
    """The same bytes as pool-shaped arrays ({gate,up,down}_{w,s})."""
    out = {}
    for proj, (o, i) in SHAPES.items():
        key = proj.split("_")[0]
        w = b"".join(fixture_bytes(proj, "weight", e, o * i // 2) for e in range(N_EXP))
        s = b"".join(fixture_bytes(proj, "weight_scale", e, o * i // 32) for e in range(N_EXP))
        out[f"{key}_w"] = np.frombuffer(w, np.uint32).reshape(N_EXP, o, i // 8)
        out[f"{key}_s"] = np.frombuffer(s, np.uint8).reshape(N_EXP, o, i // 32)
    return out


def _load(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main(ref_root: str) -> None:
    import fcntl
    conv = _load(Path(ref_root) / "scripts" / "convert-mimo-v26-mlx.py", "ref_convert")
    conv.PROJ = dict(SHAPES)

    class Index:  # the converter's SafeIndex.raw, serving the seeded bytes
        def raw(self, name):
            parts = name.split(".")           # model.layers.L.mlp.experts.E.PROJ.KIND
            e, proj, kind = int(parts[5]), parts[6], parts[7]
            o, i = SHAPES[proj]
            return bytearray(fixture_bytes(proj, kind, e, o * i // 2 if kind == "weight" else o * i // 32))

    real_fcntl = fcntl.fcntl
    fcntl.fcntl = lambda *a, **k: 0          # F_NOCACHE / F_RDAHEAD exist on macOS only
    try:
        store = _load(Path(ref_root) / "engine" / "mimo_stream" / "store.py", "ref_store")
        with tempfile.TemporaryDirectory() as d:
            path, _ = conv.convert_expert_layer(Index(), d, LAYER, N_EXP)
            blob = Path(path).read_bytes()
            st = store.ExpertStore(d, [LAYER], n_experts=N_EXP)
            loc = {f"{k}_{kind}": [st.loc[(LAYER, k, kind)][1], st.loc[(LAYER, k, kind)][2]]
                   for k in ("gate", "up", "down") for kind in ("w", "s")}
            dst = {(k, kind): memoryview(bytearray(loc[f"{k}_{kind}"][1]))
                   for k in ("gate", "up", "down") for kind in ("w", "s")}
            io = store.IOPool(2)
            io.run(st.jobs(LAYER, PROBE_EXPERT, dst))
            probe = {f"{k}_{kind}": hashlib.sha256(dst[(k, kind)]).hexdigest() for (k, kind) in dst}
            st.close()
    finally:
        fcntl.fcntl = real_fcntl
    rec = {"layer": LAYER, "n_experts": N_EXP, "shapes": SHAPES, "file_size": len(blob),
           "file_sha256": hashlib.sha256(blob).hexdigest(), "loc": loc, "probe_expert": PROBE_EXPERT,
           "probe_sha256": probe,
           "made_by": "the reference's convert_expert_layer / write_safetensors and ExpertStore / IOPool"}
    (HERE / "expert_file.json").write_text(json.dumps(rec, indent=1) + "\n")
    print(json.dumps(rec, indent=1))


if __name__ == "__main__":
    main(sys.argv[1])
