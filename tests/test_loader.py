"""Expert-file loader (mimo_moe/loader.py + the native reader) against the reference's own format code.

tests/golden/expert_file.json was recorded by tests/golden/make_expert_file.py, which ran the
reference's converter (scripts/convert-mimo-v26-mlx.py `convert_expert_layer`) and its reader
(engine/mimo_stream/store.py `ExpertStore` + `IOPool`) on seeded bytes.  Here, without the reference:
the package's writer must reproduce the converter's file byte for byte, the index must give
ExpertStore's (base, stride) for every tensor, and the native reader must return the bytes IOPool read.
The GPU tests round-trip full-size synthetic pools through a file into HBM."""
import hashlib
import json
import os

import numpy as np
import pytest
import torch

from conftest import ROOT

GOLD = json.loads((ROOT / "tests" / "golden" / "expert_file.json").read_text())


def _fixture():
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_expert_file", ROOT / "tests" / "golden" / "make_expert_file.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="module")
def expert_file(tmp_path_factory):
    from mimo_moe.loader import save_expert_file
    path = str(tmp_path_factory.mktemp("experts") / f"experts-L{GOLD['layer']:02d}.safetensors")
    save_expert_file(path, GOLD["layer"], _fixture().fixture_arrays())
    return path


def test_writer_reproduces_the_reference_converter_file(expert_file):
    blob = open(expert_file, "rb").read()
    assert len(blob) == GOLD["file_size"]
    assert hashlib.sha256(blob).hexdigest() == GOLD["file_sha256"]


def test_index_matches_the_reference_store(expert_file):
    from mimo_moe.loader import ExpertFile
    f = ExpertFile(expert_file, GOLD["layer"])
    for name, (base, stride) in GOLD["loc"].items():
        key, kind = name.split("_")
        assert (f.loc[(key, kind)].base, f.loc[(key, kind)].stride) == (base, stride), name
    assert f.num_experts == GOLD["n_experts"] and f.aligned
    assert (f.hidden, f.inter) == tuple(GOLD["shapes"]["gate_proj"][::-1])


@pytest.mark.parametrize("threads", [1, 3])
def test_native_reader_returns_the_bytes_the_reference_read(expert_file, threads):
    from mimo_moe.loader import read_expert_bytes
    e = GOLD["probe_expert"]
    got = read_expert_bytes(expert_file, GOLD["layer"], e, 1, threads=threads)
    for name, digest in GOLD["probe_sha256"].items():
        assert hashlib.sha256(got[name][0].tobytes()).hexdigest() == digest, name
    whole = read_expert_bytes(expert_file, GOLD["layer"], 1, 3, threads=threads)   # a shard [1, 4)
    ref = _fixture().fixture_arrays()
    for name, a in whole.items():
        assert np.array_equal(a.view(np.uint8), ref[name][1:4].view(np.uint8)), name


def test_chunked_reads_cross_span_boundaries(expert_file):
    """4 KiB chunks over a span that is not a chunk multiple, several threads."""
    from mimo_moe.loader import _read_spans
    size = os.path.getsize(expert_file)
    buf = np.zeros(size - 12345, np.uint8)
    _read_spans(expert_file, [(12345, buf.nbytes, buf.ctypes.data)], False, 5, 4096, False)
    assert np.array_equal(buf, np.fromfile(expert_file, np.uint8)[12345:])


def test_errors(expert_file, tmp_path):
    from mimo_moe import MimoError
    from mimo_moe.loader import ExpertFile, _read_spans, read_expert_bytes, save_expert_file
    with pytest.raises(ValueError):
        ExpertFile(expert_file, GOLD["layer"] + 1)                     # another layer's names
    with pytest.raises(ValueError):
        read_expert_bytes(expert_file, GOLD["layer"], 3, 2)          # past the last expert
    short = tmp_path / "short.safetensors"
    short.write_bytes(open(expert_file, "rb").read()[:-4096])
    with pytest.raises(ValueError):
        ExpertFile(str(short), GOLD["layer"])                        # ranges beyond the file
    buf = np.zeros(8192, np.uint8)
    with pytest.raises(MimoError) as ei:
        _read_spans(str(short), [(os.path.getsize(short) - 4096, 8192, buf.ctypes.data)], False, 2, 4096, False)
    assert ei.value.code == 5                                          # MIMO_EIO: short read
    with pytest.raises(MimoError):
        _read_spans(str(tmp_path / "missing"), [(0, 16, buf.ctypes.data)], False, 1, 4096, False)
    bad = _fixture().fixture_arrays()
    bad["up_s"] = bad["up_s"][:, :, :-1]                               # 31 values per scale
    save_expert_file(str(tmp_path / "bad.safetensors"), 0, bad)
    with pytest.raises(ValueError):
        ExpertFile(str(tmp_path / "bad.safetensors"), 0)


@pytest.mark.gpu
def test_full_size_pool_round_trip_and_shard(gpu, tmp_path):
    import mimo_moe
    from mimo_moe.loader import ExpertFile, load_expert_pools, save_expert_file
    src = mimo_moe.ExpertPools.synthetic(8, seed=0, layer=7, device=gpu)
    path = str(tmp_path / "experts-L07.safetensors")
    save_expert_file(path, 7, src.t)
    f = ExpertFile(path, 7)
    assert f.aligned and (f.hidden, f.inter, f.num_experts) == (4096, 2048, 8)
    for threads, chunk, direct in ((8, 16 << 20, True), (3, 1 << 20, False)):
        got = load_expert_pools(path, 7, device=gpu, threads=threads, chunk_bytes=chunk, direct=direct)
        for name, t in src.t.items():
            assert torch.equal(got.t[name], t), name
    shard = load_expert_pools(path, 7, first_expert=3, count=2, device=gpu)
    for name, t in src.t.items():
        assert torch.equal(shard.t[name], t[3:5]), name
    x = torch.randn(2, 4096, device=gpu).to(torch.bfloat16)
    W = (torch.randn(32, 4096, device=gpu) * 0.02).to(torch.bfloat16)
    big = mimo_moe.ExpertPools.synthetic(32, seed=0, layer=7, device=gpu)
    save_expert_file(path, 7, big.t)
    loaded = load_expert_pools(path, 7, device=gpu)
    y0 = mimo_moe.moe_block(x, W, None, big)
    y1 = mimo_moe.moe_block(x, W, None, loaded)
    assert torch.equal(y0.view(torch.int16), y1.view(torch.int16))


@pytest.mark.gpu
def test_router_from_dense_file(gpu, tmp_path):
    import struct
    from mimo_moe.loader import load_router
    W = (torch.randn(256, 4096) * 0.02).to(torch.bfloat16)
    b = torch.randn(256)
    names = {"model.layers.3.mlp.gate.weight": ("BF16", W.view(torch.int16).numpy()),
             "model.layers.3.mlp.gate.e_score_correction_bias": ("F32", b.numpy())}
    hdr, off, blobs = {}, 0, []
    for n, (dt, a) in names.items():
        hdr[n] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        off += a.nbytes
        blobs.append(a.tobytes())
    hj = json.dumps(hdr).encode()
    p = tmp_path / "dense.safetensors"
    p.write_bytes(struct.pack("<Q", len(hj)) + hj + b"".join(blobs))
    W2, b2 = load_router(str(p), 3, device=gpu)
    assert torch.equal(W2.cpu().view(torch.int16), W.view(torch.int16)) and torch.equal(b2.cpu(), b)
