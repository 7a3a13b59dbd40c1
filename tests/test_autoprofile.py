from pathlib import Path

from teamredbench_b200.config import load_suite
from teamredbench_b200.device import DeviceInfo
from teamredbench_b200.runner import build_context

SUITES = Path(__file__).resolve().parent.parent / "teamredbench_b200" / "configs" / "suites"


def test_build_context_auto_selects_b200_profile(monkeypatch):
    suite = load_suite(SUITES / "smoke.yaml")
    monkeypatch.setattr("teamredbench_b200.runner.load_torch", lambda: None)
    monkeypatch.setattr("teamredbench_b200.runner.detect_device",
                        lambda torch_module, device_id=0: DeviceInfo(index=device_id, name="NVIDIA B200"))
    context, note = build_context(suite, device_id=0)
    assert context.hardware_profile.name == "nvidia-b200"
    assert note is not None and "B200" in note


def test_unknown_device_keeps_placeholder(monkeypatch):
    suite = load_suite(SUITES / "smoke.yaml")
    monkeypatch.setattr("teamredbench_b200.runner.load_torch", lambda: None)
    monkeypatch.setattr("teamredbench_b200.runner.detect_device",
                        lambda torch_module, device_id=0: DeviceInfo(index=device_id, name="Some GPU"))
    context, note = build_context(suite, device_id=0)
    assert context.hardware_profile.name == "nvidia-generic" and note is None
