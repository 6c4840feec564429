"""Mode routing: the b200 mode builds a B200Engine; unknown modes fail first."""
import sys
from types import SimpleNamespace

import pytest

from laya_b200.modes import create_engine


def test_unknown_mode_fails_before_loading_anything():
    with pytest.raises(ValueError, match="mode must be balanced, fast or b200"):
        create_engine(mode="typo")


def test_b200_mode_builds_b200_engine(monkeypatch):
    made = []
    monkeypatch.setitem(sys.modules, "laya_b200.engine",
                        SimpleNamespace(B200Engine=lambda **kw: made.append(kw) or "engine"))
    assert create_engine(mode="b200", precision="fp8", device="cuda:1") == "engine"
    assert made == [{"precision": "fp8", "device": "cuda:1"}]


def test_reference_modes_need_the_reference_package(monkeypatch):
    monkeypatch.setitem(sys.modules, "laya_blackwell", None)
    monkeypatch.setitem(sys.modules, "laya_blackwell.modes", None)
    with pytest.raises(RuntimeError, match="laya_blackwell"):
        create_engine(mode="balanced")
