"""Property tests of the native PEFT packer (plora_peft_pack) against the
Python loader, which follows the reference (src/polylora/store.py:304-388) and
reads files with safetensors' own loader.

The packer may decline any file (the Python path then loads it or raises);
when it accepts one, the Python path must accept it too and load the same
weights.  Files are written by hand so that the header order, gaps between
data blocks, trailing bytes and number literals can differ from what
safetensors itself writes."""

import json
import tempfile
from pathlib import Path

import pytest
import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from polylora_b200.store import CpuAdapterStore

# module name -> (in_features, out_features); names that are string suffixes of
# one another exercise the reference's key matching
POOL = {"q": (3, 3), "attn.q": (3, 3), "layer.1.dense": (4, 6), "encoder.layer.1.dense": (4, 6),
        "layer.11.dense": (5, 3)}
CODES = {torch.bfloat16: "BF16", torch.float32: "F32"}


def write_safetensors(path: Path, entries, header_order=None, gap_after=None, trailing=0, float_shape=None,
                      metadata=None):
    """entries: (key, tensor) in data order.  header_order: key order of the
    JSON header; gap_after: index of the block followed by 8 unused bytes;
    float_shape: key whose shape is written with float literals."""
    data, header = b"", {}
    for i, (key, t) in enumerate(entries):
        blob = t.contiguous().view(-1).view(torch.uint8).numpy().tobytes()
        header[key] = {"dtype": CODES[t.dtype], "shape": list(t.shape), "data_offsets": [len(data), len(data) + len(blob)]}
        data += blob
        if gap_after == i:
            data += bytes(8)
    data += bytes(trailing)
    ordered = {"__metadata__": metadata} if metadata is not None else {}
    for key in header_order or list(header):
        ordered[key] = header[key]
    raw = json.dumps(ordered)
    if float_shape is not None:
        shape = ordered[float_shape]["shape"]
        raw = raw.replace(json.dumps({"shape": shape})[1:-1], json.dumps({"shape": [float(d) for d in shape]})[1:-1], 1)
    raw = raw.encode()
    raw += b" " * (-len(raw) % 8)
    path.write_bytes(len(raw).to_bytes(8, "little") + raw + data)


@st.composite
def peft_files(draw):
    names = draw(st.lists(st.sampled_from(sorted(POOL)), min_size=1, max_size=4, unique=True))
    adapter = draw(st.sampled_from(["default", "other"]))
    g = torch.Generator().manual_seed(draw(st.integers(0, 1000)))
    entries = []
    for m in sorted(POOL):
        k_in, n_out = POOL[m]
        # mostly one key pair per configured module and none for the others,
        # so that most files load; extra pairs compete for the first match
        pairs = draw(st.sampled_from([1, 1, 1, 1, 2, 0] if m in names else [0] * 8 + [1]))
        for _ in range(pairs):
            prefix = draw(st.sampled_from(["base_model.model.", "base_model.model.x.", ""]))
            infix = draw(st.sampled_from([".", ".default.", ".other."]))
            r = draw(st.integers(1, 3))
            rb = r + 1 if draw(st.integers(0, 19)) == 0 else r  # sometimes inconsistent ranks
            dt_a = torch.float32 if draw(st.integers(0, 19)) == 0 else torch.bfloat16
            dt_b = torch.float32 if draw(st.integers(0, 19)) == 0 else torch.bfloat16
            side = draw(st.sampled_from(["both"] * 8 + ["a", "b"]))
            if side in ("both", "a"):
                entries.append((f"{prefix}{m}.lora_A{infix}weight", torch.randn(r, k_in, generator=g).to(dt_a)))
            if side in ("both", "b"):
                entries.append((f"{prefix}{m}.lora_B{infix}weight", torch.randn(n_out, rb, generator=g).to(dt_b)))
    if draw(st.booleans()):
        entries.append(("unrelated.weight", torch.randn(2, 2, generator=g).to(torch.bfloat16)))
    entries = [e for i, e in enumerate(entries) if e[0] not in {k for k, _ in entries[:i]}]  # unique keys
    entries = draw(st.permutations(entries))  # data order
    header_order = [k for k, _ in draw(st.permutations(entries))] if draw(st.booleans()) else None
    defect = draw(st.sampled_from(["none"] * 6 + ["gap", "trailing", "float_shape", "bad_metadata"]))
    alpha = draw(st.sampled_from([1.0, 4.0, 6.5]))
    return names, adapter, entries, header_order, defect, alpha


def _write_adapter(root: Path, entries, header_order, defect, alpha) -> Path:
    root.mkdir(parents=True, exist_ok=True)
    (root / "adapter_config.json").write_text(json.dumps({"peft_type": "LORA", "r": 3, "lora_alpha": alpha}))
    kw = {}
    if defect == "gap" and len(entries) > 1:
        kw["gap_after"] = 0
    elif defect == "trailing":
        kw["trailing"] = 8
    elif defect == "float_shape" and entries:
        kw["float_shape"] = entries[0][0]
    elif defect == "bad_metadata":
        kw["metadata"] = {"format": 1}
    write_safetensors(root / "adapter_model.safetensors", entries, header_order, **kw)
    return root


def _general(store, path: Path, names, adapter):
    try:
        config, state_dict = store._read_peft_dir(path)
        return store._layers_from_peft_state_dict("x", state_dict, names, float(config["lora_alpha"]), adapter)
    except Exception as exc:  # noqa: BLE001 - any refusal of the reference's path
        return exc


def _assert_same_layers(packed, general):
    assert not isinstance(general, Exception), f"packer accepted a file the Python path rejects: {general!r}"
    assert packed.keys() == general.keys()
    for m, w in packed.items():
        v = general[m]
        assert (w.rank, w.scale, w.A.dtype) == (v.rank, v.scale, v.A.dtype)
        assert torch.equal(w.A, v.A) and torch.equal(w.B, v.B)


@settings(max_examples=300, deadline=None, derandomize=True, suppress_health_check=list(HealthCheck))
@given(peft_files())
def test_packer_accepts_only_what_the_python_path_loads_identically(case):
    names, adapter, entries, header_order, defect, alpha = case
    with tempfile.TemporaryDirectory() as d:
        path = _write_adapter(Path(d) / "a", entries, header_order, defect, alpha)
        store = CpuAdapterStore(module_names=names)
        store.set_image_spec(names, torch.bfloat16)
        packed = store._load_direct("x", path, names, adapter)
        general = _general(store, path, names, adapter)
        if packed is not None:
            assert defect == "none", f"packer accepted a file with defect {defect}"
            _assert_same_layers(packed[1], general)


def test_packer_takes_the_first_key_in_data_order_not_header_order(tmp_path):
    """Two keys match module 'attn.q'; the header lists them in the opposite
    order of their data blocks.  safetensors' load_file returns keys in data
    order, so the reference uses the first data block: so must the packer."""
    g = torch.Generator().manual_seed(5)
    t = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16)  # noqa: E731
    entries = [("base_model.model.x.attn.q.lora_A.weight", t(2, 3)), ("base_model.model.x.attn.q.lora_B.weight", t(3, 2)),
               ("base_model.model.attn.q.lora_A.weight", t(3, 3)), ("base_model.model.attn.q.lora_B.weight", t(3, 3))]
    path = _write_adapter(tmp_path / "a", entries, [k for k, _ in reversed(entries)], "none", 4.0)
    store = CpuAdapterStore(module_names=["attn.q"])
    store.set_image_spec(["attn.q"], torch.bfloat16)
    packed = store._load_direct("x", path, ["attn.q"], "default")
    assert packed is not None
    _assert_same_layers(packed[1], _general(store, path, ["attn.q"], "default"))
    assert packed[1]["attn.q"].rank == 2  # the first data block's pair


@pytest.mark.parametrize("seed", range(4))
def test_packer_survives_mutated_headers(tmp_path, seed):
    """Random bytes of a valid file's header overwritten: the packer returns a
    status and never crashes; a file it still accepts loads as the Python
    path loads it."""
    import ctypes

    from polylora_b200 import _native

    lib = _native.load()
    names = ["attn.q", "layer.1.dense"]
    g = torch.Generator().manual_seed(seed)
    entries = []
    for m in names:
        k_in, n_out = POOL[m]
        entries += [(f"base_model.model.{m}.lora_A.weight", torch.randn(2, k_in, generator=g).to(torch.bfloat16)),
                    (f"base_model.model.{m}.lora_B.weight", torch.randn(n_out, 2, generator=g).to(torch.bfloat16))]
    src = _write_adapter(tmp_path / "src", entries, None, "none", 4.0)
    good = (src / "adapter_model.safetensors").read_bytes()
    hlen = int.from_bytes(good[:8], "little")
    c_names = (ctypes.c_char_p * len(names))(*[n.encode() for n in names])
    dims = (ctypes.c_int64 * (3 * len(names)))()
    nbytes = ctypes.c_size_t(0)
    image = torch.empty(1 << 16, dtype=torch.uint8)
    rng = torch.Generator().manual_seed(100 + seed)
    store = CpuAdapterStore(module_names=names)
    store.set_image_spec(names, torch.bfloat16)
    accepted = 0
    for i in range(150):
        raw = bytearray(good)
        for _ in range(1 + i % 4):
            pos = 8 + int(torch.randint(0, hlen, (1,), generator=rng))
            raw[pos] = int(torch.randint(32, 127, (1,), generator=rng))
        path = tmp_path / f"m{i}"
        path.mkdir()
        (path / "adapter_config.json").write_text((src / "adapter_config.json").read_text())
        (path / "adapter_model.safetensors").write_bytes(bytes(raw))
        st_ = lib.plora_peft_pack(str(path / "adapter_model.safetensors").encode(), c_names, len(names), b"default",
                                  2, 4.0, image.data_ptr(), image.numel(), ctypes.byref(nbytes), dims)
        assert st_ in (_native.OK, _native.ERR_UNSUPPORTED), st_
        if st_ == _native.OK:
            accepted += 1
            packed = store._load_direct("x", path, names, "default")
            assert packed is not None
            _assert_same_layers(packed[1], _general(store, path, names, "default"))
    assert accepted < 150  # the mutations did change what the packer sees
