"""PrecisionConfig mirror: the reference's tests/test_precision.py, plus the real FP8 preset."""
import dataclasses

import pytest

from whisper_blaze_b200.precision import (LayerPrecision, Precision, PrecisionConfig, aggressive_fp8, fp8_e4m3,
                                          from_name, full_fp16, mixed_fp8)


def test_is_fp8():
    assert not Precision.FP16.is_fp8()
    assert Precision.FP8_E4M3.is_fp8() and Precision.FP8_E5M2.is_fp8()


def test_max_val():
    assert Precision.FP16.max_val() == 65504.0
    assert Precision.FP8_E4M3.max_val() == 448.0
    assert Precision.FP8_E5M2.max_val() == 57344.0


def test_layer_precision():
    assert not LayerPrecision().is_fp8()
    assert LayerPrecision(Precision.FP8_E4M3, Precision.FP8_E4M3).is_fp8()
    assert LayerPrecision(Precision.FP8_E4M3, Precision.FP8_E5M2).is_fp8()


def test_full_fp16_all_fp16():
    for name, lp in full_fp16().__dict__.items():
        assert lp.weight == Precision.FP16 and lp.activation == Precision.FP16, name


def test_deprecated_presets_still_alias_fp16():
    for preset in (mixed_fp8, aggressive_fp8):
        with pytest.deprecated_call():
            cfg = preset()
        assert cfg == full_fp16()
        for f in dataclasses.fields(cfg):
            assert not getattr(cfg, f.name).is_fp8()


def test_real_fp8_preset():
    cfg = from_name("fp8_e4m3")
    assert cfg == fp8_e4m3()
    for f in dataclasses.fields(cfg):
        lp = getattr(cfg, f.name)
        assert lp.weight == Precision.FP8_E4M3 and lp.activation == Precision.FP8_E4M3
    assert Precision.FP8_E4M3.fmt() == "e4m3" and Precision.FP8_E5M2.fmt() == "e5m2"


def test_from_name():
    assert isinstance(from_name("fp16"), PrecisionConfig)
    assert not from_name("mixed_fp8").encoder_ffn.weight.is_fp8()
    with pytest.raises(ValueError, match="Unknown precision preset"):
        from_name("nonexistent_preset")


def test_summary_str():
    s = full_fp16().summary()
    assert "PrecisionConfig" in s and "encoder_ffn" in s
