"""Export directories on the host: which model a directory holds and the checks of an export, as the reference's
loader makes them (src/kea_kernels/formats.py:95-172) - no GPU."""
from __future__ import annotations

import json

import pytest

from fake_export import write_export
from kea_kernels import formats


@pytest.mark.parametrize("kind,model,mode", [("binary", "kea-b", "x2"), ("ternary", "kea-t", "x2")])
def test_describe_and_check_a_valid_export(tmp_path, kind, model, mode):
    d = write_export(tmp_path / "m", kind, encoder_tensors=False)
    md = formats.describe(d)
    assert (md.model, md.kind, md.default_mode) == (model, kind, mode)
    manifest = formats.check_export(d, kind)
    assert len(manifest["quantized_layers"]) == formats.EXPECTED_MODULES
    with pytest.raises(ValueError, match="format"):
        formats.check_export(d, "ternary" if kind == "binary" else "binary")


def test_kea_b_0_1_bundle_reads_its_compat_export(tmp_path):
    root = tmp_path / "kea-b-0.1"
    root.mkdir()
    (root / formats.MANIFEST).write_text(json.dumps({"format": formats.BUNDLE_FORMAT, "sha256": "abc"}))
    write_export(root / formats.COMPAT_DIR, "binary", encoder_tensors=False, extra={"keab": {"bundle_sha256": "abc"}})
    md = formats.describe(root)
    assert (md.model, md.kind, md.default_mode) == ("kea-b-0.1", "binary", "x1")
    assert md.export_dir == (root / formats.COMPAT_DIR).resolve()
    (root / formats.MANIFEST).write_text(json.dumps({"format": formats.BUNDLE_FORMAT, "sha256": "other"}))
    with pytest.raises(ValueError, match="does not record"):
        formats.describe(root)


def test_describe_rejects_unknown_directories(tmp_path):
    with pytest.raises(ValueError, match="no manifest.json"):
        formats.describe(tmp_path)
    (tmp_path / formats.MANIFEST).write_text(json.dumps({"format": "something-else"}))
    with pytest.raises(ValueError, match="unsupported format"):
        formats.describe(tmp_path)
    (tmp_path / formats.MANIFEST).write_text(json.dumps({"format": formats.BUNDLE_FORMAT, "sha256": "x"}))
    with pytest.raises(ValueError, match="without its compat"):
        formats.describe(tmp_path)


def test_a_modified_file_fails_the_sha256_check(tmp_path):
    d = write_export(tmp_path / "m", "binary", encoder_tensors=False)
    (d / "tokenizer" / "vocab.txt").write_text("changed\n")
    with pytest.raises(ValueError, match="SHA-256"):
        formats.check_export(d, "binary")
    formats.check_export(d, "binary", verify_hashes=False)


def _drop_first_layer(layers, tensors):
    name = next(iter(layers))
    del layers[name]


def _dense_weight(layers, tensors):
    name = next(iter(layers))
    tensors[f"{name}.weight"] = tensors[f"{name}.scale"].clone()


def _wrong_codes_shape(layers, tensors):
    name = next(iter(layers))
    tensors[f"{name}.codes"] = tensors[f"{name}.codes"][:, :-1].contiguous()


def _bias_flag(layers, tensors):
    name = next(n for n in layers if not layers[n]["bias"])
    layers[name]["bias"] = True


def _bad_kind(layers, tensors):
    layers[next(iter(layers))]["kind"] = "conv2d"


def _bad_name(layers, tensors):
    name = next(iter(layers))
    layers[name.replace("linear1", "linear9")] = layers.pop(name)


@pytest.mark.parametrize("tamper,match", [(_drop_first_layer, "264"), (_dense_weight, "dense weight"),
                                          (_wrong_codes_shape, "codes must be"), (_bias_flag, "bias presence"),
                                          (_bad_kind, "unknown kind"), (_bad_name, "264")])
def test_check_export_rejects_malformed_exports(tmp_path, tamper, match):
    d = write_export(tmp_path / "m", "ternary", encoder_tensors=False, tamper=tamper)
    with pytest.raises(ValueError, match=match):
        formats.check_export(d, "ternary")


def test_check_export_rejects_a_wrong_model_target(tmp_path):
    d = write_export(tmp_path / "m", "binary", encoder_tensors=False)
    manifest = json.loads((d / formats.MANIFEST).read_text())
    manifest["config"]["target"] = "some.other.Model"
    (d / formats.MANIFEST).write_text(json.dumps(manifest))
    with pytest.raises(ValueError, match="model target"):
        formats.check_export(d, "binary")
