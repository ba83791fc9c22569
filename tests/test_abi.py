"""The C-ABI boundary without a GPU: the library loads, exports every function the
public headers declare, and rejects bad configurations with the reference's messages
before touching a device; the KV page swizzle helper is an exact involution."""
import re

import numpy as np
import pytest

from conftest import ROOT


def _declared_functions():
    names = set()
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"//[^\n]*", "", text)
        for m in re.finditer(r"(?:^|[;}\n])\s*(?:const\s+)?[A-Za-z_][A-Za-z0-9_]*[\s*]+(qasr_[a-z0-9_]+)\s*\(",
                             text):
            names.add(m.group(1))
    return names


def test_headers_declare_what_the_package_lists(qasr):
    declared = _declared_functions()
    assert len(declared) > 30
    assert declared == set(qasr.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_function(qasr):
    missing = [n for n in sorted(_declared_functions()) if not hasattr(qasr.lib, n)]
    assert not missing, missing


def test_version_string(qasr):
    assert qasr.version().startswith("qasr_b200")


@pytest.mark.parametrize("change,needle", [
    (dict(head_dim=64), "head_dim must be 128"),
    (dict(num_attention_heads=24), "2 query heads per kv head"),
    (dict(hidden_size=1000), "multiples of 128"),
    (dict(vocab_size=151937), "multiples of 128"),
])
def test_create_rejects_unsupported_configs(qasr, change, needle):
    cfg = dict(qasr.text_config("0.6b"))
    cfg.update(change)
    with pytest.raises(qasr.DecoderError) as e:
        qasr.TextDecoder(cfg)
    assert e.value.status == 1 and needle in str(e.value)


def test_create_rejects_bad_options(qasr):
    cfg = qasr.text_config("0.6b")
    with pytest.raises(qasr.DecoderError) as e:
        qasr.TextDecoder(cfg, weight_format=7)
    assert "weight_format" in str(e.value)
    with pytest.raises(qasr.DecoderError) as e:
        qasr.TextDecoder(cfg, max_slots=0)
    assert "max_slots" in str(e.value)
    # 64 slots x (2^31 - 1) positions: 2^31 page-table entries, refused before any
    # allocation instead of wrapping the 32-bit page count
    with pytest.raises(qasr.DecoderError) as e:
        qasr.TextDecoder(cfg, max_slots=64, max_seq=2**31 - 1)
    assert e.value.status == 1 and "32-bit page indices" in str(e.value)


def test_kv_page_swizzle_is_an_involution(qasr):
    rng = np.random.default_rng(0)
    pool = rng.integers(0, 65535, size=(3, 2, 2, 4, 64, 128), dtype=np.uint16)
    sw = qasr.kv_page_swizzle(pool)
    np.testing.assert_array_equal(qasr.kv_page_swizzle(sw), pool)
    # dim d of position p lands at column ((d // 8) ^ (p % 8)) * 8 + d % 8
    for p, d in [(0, 0), (1, 0), (7, 127), (9, 13), (63, 64)]:
        col = (((d // 8) ^ (p % 8)) * 8) + d % 8
        assert sw[1, 0, 1, 2, p, col] == pool[1, 0, 1, 2, p, d]


@pytest.mark.parametrize("preset", ["0.6b", "1.7b"])
@pytest.mark.parametrize("fmt", ["f16", "int8", "int8_f32"])
def test_layer_sizes_match_the_loader_inputs(qasr, preset, fmt):
    """qasr_load_layer reads each field as `count` values of `itemsize` bytes; the Python
    mirror refuses arrays of another size (layer_sizes).  The synthetic layers the tests and
    the bench load — and the rope tables — have exactly those sizes in every format."""
    cfg = qasr.text_config(preset, num_hidden_layers=1, vocab_size=1024)
    wf = {"f16": qasr.WEIGHTS_F16, "int8": qasr.WEIGHTS_INT8, "int8_f32": qasr.WEIGHTS_INT8_F32}[fmt]
    sizes = qasr.layer_sizes(cfg, wf)
    layer = qasr.SyntheticModel(cfg, seed=3).layer(0, int8=fmt != "f16", scale_f32=fmt == "int8_f32")
    for name, a in layer.items():
        if name.endswith("_scale") and fmt == "f16":
            continue
        assert (a.size, a.itemsize) == sizes[name], name
    assert {n for n in sizes if fmt != "f16" or not n.endswith("_scale")} == set(layer)
    with pytest.raises(ValueError, match="q_proj"):
        qasr._sized("q_proj", layer["q_proj"][:-1], *sizes["q_proj"])
    cos, sin = qasr.build_rope_tables(64)
    assert cos.shape == sin.shape == (64, cfg["head_dim"]) and cos.itemsize == 2
