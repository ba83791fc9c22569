"""The host-side parsers fed garbage: config.json text and safetensors headers that are
random, truncated or structurally wrong must come back as a status code and a message,
never a crash (they run inside the caller's process).  Seeded, a few hundred cases each."""
import json
import struct

import numpy as np

from safetensors_io import write_safetensors


def _json_cases(rng):
    good = json.dumps({"thinker_config": {"text_config": {"hidden_size": 1024}, "audio_config": {"d_model": 896}}})
    yield ""
    yield "{"
    yield "[" * 5000  # deep nesting
    yield '{"thinker_config": ' * 3000
    yield '{"a": "\\u12"}'
    yield '{"text_config": {"hidden_size": 1e309}}'
    yield '{"text_config": {"hidden_size": 99999999999999999999999}}'
    for _ in range(300):
        b = bytearray(good.encode())
        for _ in range(int(rng.integers(1, 8))):
            i = int(rng.integers(0, len(b)))
            op = int(rng.integers(0, 3))
            if op == 0:
                b[i] = int(rng.integers(0, 256))
            elif op == 1:
                del b[i]
            else:
                b[i:i] = bytes([int(rng.integers(32, 127))])
        yield bytes(b).decode("latin-1")
    for _ in range(100):
        yield bytes(rng.integers(0, 256, int(rng.integers(0, 200)), dtype=np.uint8)).decode("latin-1")


def test_config_parsers_survive_garbage(qasr, tmp_path):
    rng = np.random.default_rng(1234)
    d = tmp_path / "m"
    d.mkdir()
    n_ok = 0
    for text in _json_cases(rng):
        (d / "config.json").write_bytes(text.encode("latin-1"))
        for fn in (qasr.read_model_config, qasr.read_audio_config):
            try:
                fn(str(d))
                n_ok += 1
            except qasr.DecoderError as e:
                assert e.status == 1
    assert n_ok > 0  # some mutations leave a valid file


def test_checkpoint_open_survives_bad_headers(qasr, tmp_path):
    rng = np.random.default_rng(99)
    good = tmp_path / "good.safetensors"
    write_safetensors(good, {"model.language_model.norm.weight": np.ones(8, np.float16)})
    raw = good.read_bytes()
    hlen = struct.unpack("<Q", raw[:8])[0]
    cases = [b"", raw[:7], struct.pack("<Q", 1 << 60) + raw[8:], struct.pack("<Q", hlen + 100) + raw[8:],
             raw[:8 + hlen // 2]]
    for _ in range(200):
        b = bytearray(raw)
        for _ in range(int(rng.integers(1, 6))):
            i = int(rng.integers(0, 8 + hlen))
            b[i] = int(rng.integers(0, 256))
        cases.append(bytes(b))
    opened = 0
    for k, blob in enumerate(cases):
        d = tmp_path / f"c{k}"
        d.mkdir()
        (d / "model.safetensors").write_bytes(blob)
        try:
            with qasr.Checkpoint(str(d)) as ck:
                opened += 1
                for name in ("model.language_model.norm.weight", "thinker.model.norm.weight"):
                    try:
                        ck.read_f32(name)
                    except qasr.DecoderError:
                        pass
        except qasr.DecoderError as e:
            assert e.status in (1, 2)
    assert opened >= 1


def _raw_safetensors(header: dict, data: bytes) -> bytes:
    h = json.dumps(header).encode()
    return struct.pack("<Q", len(h)) + h + data


def test_checkpoint_rejects_shapes_whose_product_wraps(qasr, tmp_path):
    """A shape product that overflows 64 bits (or the byte size) must be rejected when the
    file is opened: wrapped to a small element count, it would pass the size check and
    let a row read run past the mapped file."""
    cases = {
        "wraps_to_zero": {"dtype": "F16", "shape": [1 << 33, 1 << 31], "data_offsets": [0, 0]},
        "wraps_bytes": {"dtype": "F32", "shape": [1 << 62, 4], "data_offsets": [0, 0]},
        "huge_rows": {"dtype": "I8", "shape": [1 << 40, 1 << 30], "data_offsets": [0, 16]},
    }
    for k, (name, entry) in enumerate(cases.items()):
        d = tmp_path / f"w{k}"
        d.mkdir()
        (d / "model.safetensors").write_bytes(_raw_safetensors({"thinker.model.norm.weight": entry}, bytes(16)))
        try:
            with qasr.Checkpoint(str(d)) as ck:
                raise AssertionError(f"{name}: opened a checkpoint with {len(ck)} tensors")
        except qasr.DecoderError as e:
            assert e.status == 1, name
            assert "overflow" in str(e) or "bytes" in str(e), (name, str(e))
