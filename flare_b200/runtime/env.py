"""Runtime environment presets for one-process-per-GPU training over NCCL/NVLink.

``distributed_env(existing)`` returns the environment a training process
should start with: the NCCL, allocator and launcher settings this framework
is tuned for, merged with what the caller already set.  A caller value that
contradicts a preset raises (the reference's rule for its XLA flag preset,
src/flare/jax/xla_preset.py:6-34); ``overrides`` replaces presets on purpose.
``fault_test_env`` is the variant for multi-GPU failure tests: NVLS off, so no
rank's memory is bound to an NVLink multicast object when a peer goes away.
``runtime_env`` builds the per-worker env dict (PYTHONPATH to this package)
that the reference builds for its JAX workers (src/flare/jax/runtime_env.py:12).
"""
from __future__ import annotations

from collections.abc import Mapping
from pathlib import Path

DISTRIBUTED_PRESET: Mapping[str, str] = {
    # the fused kernels exchange through peer memory; NCCL is used for the plain collectives around them
    "NCCL_P2P_LEVEL": "NVL",
    "NCCL_NVLS_ENABLE": "1",                   # NVSwitch in-switch reductions for the NCCL all-reduces
    "TORCH_NCCL_AVOID_RECORD_STREAMS": "1",
    "TORCH_NCCL_ASYNC_ERROR_HANDLING": "3",    # a failed collective tears the process down (no silent hang)
    "CUDA_DEVICE_MAX_CONNECTIONS": "32",       # side streams (host-tier copies, prefetch) overlap the main one
    "PYTORCH_CUDA_ALLOC_CONF": "expandable_segments:True",
    "OMP_NUM_THREADS": "4",
}

FAULT_TEST_PRESET: Mapping[str, str] = {**DISTRIBUTED_PRESET, "NCCL_NVLS_ENABLE": "0"}


def merge_preset(preset: Mapping[str, str], existing: Mapping[str, str] | None = None, *,
                 overrides: Mapping[str, str] | None = None) -> dict[str, str]:
    """``existing`` + ``preset``; a different existing value for a preset key raises unless overridden."""
    env = dict(existing or {})
    over = dict(overrides or {})
    for k, v in preset.items():
        if k in over:
            continue
        if k in env and env[k] != v:
            raise ValueError(f"environment variable {k}={env[k]!r} conflicts with the preset value {v!r}")
        env[k] = v
    env.update(over)
    return env


def distributed_env(existing: Mapping[str, str] | None = None, **kw) -> dict[str, str]:
    return merge_preset(DISTRIBUTED_PRESET, existing, **kw)


def fault_test_env(existing: Mapping[str, str] | None = None, **kw) -> dict[str, str]:
    return merge_preset(FAULT_TEST_PRESET, existing, **kw)


def runtime_env(*, extra: Mapping[str, str] | None = None, fault_test: bool = False,
                peer_timeout_s: float | None = None) -> dict[str, dict[str, str]]:
    """Env dict for a worker process: presets, this package on PYTHONPATH, optional peer-wait timeout."""
    env = (fault_test_env if fault_test else distributed_env)(extra)
    root = Path(__file__).resolve().parents[2]
    env["PYTHONPATH"] = str(root)
    if peer_timeout_s is not None:
        if peer_timeout_s <= 0:
            raise ValueError("peer_timeout_s must be positive")
        env["FLARE_PEER_TIMEOUT_S"] = str(peer_timeout_s)
    return {"env_vars": env}


if __name__ == "__main__":  # print shell exports of the preset
    import os

    for k, v in distributed_env({k: os.environ[k] for k in DISTRIBUTED_PRESET if k in os.environ}).items():
        print(f"export {k}={v}")


__all__ = ["DISTRIBUTED_PRESET", "FAULT_TEST_PRESET", "distributed_env", "fault_test_env", "merge_preset",
           "runtime_env"]
