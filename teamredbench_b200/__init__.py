"""TeamRedBench B200 backend.

Host-side mirror of the reference's plugin API (benchmark / metric /
native-kernel / profiler registries, YAML profiles, JSON+CSV+metadata output)
over libtrb_b200.so, the hand-written sm_100a kernels behind the `hbm` and
`mfu` benchmarks.  `collective` stays on torch.distributed + NCCL."""
__all__ = ["__version__"]

__version__ = "0.1.0"
