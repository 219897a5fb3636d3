"""fastembed_b200 — B200 (sm_100a) encoder forward path with fastEmbed's op and
model API: hand-written tcgen05/TMA kernels behind a C ABI
(include/fastembed_b200.h), host runtime in C++, Python bindings for tests and
benchmarks."""
from . import capi, workload  # noqa: F401

__all__ = ["capi", "workload"]
