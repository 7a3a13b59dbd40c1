from types import SimpleNamespace

from teamredbench_b200.device import detect_runtime, rocm_device_available


def test_detect_runtime_reports_cuda_fields(monkeypatch):
    monkeypatch.setattr("teamredbench_b200.device._run_command", lambda command: None)
    torch_module = SimpleNamespace(__version__="2.11.0", version=SimpleNamespace(hip=None, cuda="12.8"))
    runtime = detect_runtime(torch_module)
    assert runtime["torch"]["torch_version"] == "2.11.0"
    assert runtime["torch"]["cuda_version"] == "12.8"
    assert runtime["nvidia_smi"] is None


def test_reference_helper_aliases():
    fake = SimpleNamespace(cuda=SimpleNamespace(is_available=lambda: True))
    assert rocm_device_available(fake) is True
    assert rocm_device_available(None) is False
