"""A precision profile for the reference's C3.2 -> C3.4 planning path.

The reference scheduler hard-codes ``Strategy(mode=FULL_FP32)``
(c34/scheduler.py:70), so every ``KernelStep.precision_profile`` it emits says
fp32 and its MIXED policy (c32/strategy.py:76-158) is never reached from a
plan.  ``B200Scheduler`` is the reference ``ExecutionScheduler`` with one
change: its strategy selects ``profile`` ("bf16" or "fp16", fp32
accumulation) for the contraction nodes the B200 backend runs on tensor
cores -- the fused nodes of ``c33_passes`` and ``FusedGemmEpilogue`` -- and
keeps the reference's rules for everything else (sensitive ops stay fp32).
The per-node choice flows through ``select_precision`` / ``decompose``
(c34/scheduler.py:173-192) into ``KernelStep.precision_profile``
(c34/execution_plan.py:65), where the native plan runner reads it.

This module needs the reference package on ``sys.path`` (plan building happens
where the reference is installed); the plans it produces are plain data
(``c34_plan.plan_to_dict``) and replay without it.
"""

from __future__ import annotations

from typing import Any

# Node types whose contraction runs on tcgen05 when the profile asks for a
# 16-bit format.
TENSOR_CORE_OPS = {"B200ConvBiasAct", "B200LinearEpilogue", "B200FlashAttention", "FusedGemmEpilogue"}
PROFILES = ("fp32", "bf16", "fp16")


def b200_hardware():
    """HardwareCapability of one B200 (sm_100a): 227 KB of shared memory per
    block, 228 KB per SM, bf16/fp16/fp8/fp4 tensor cores."""
    from c32.hardware import HardwareCapability
    return HardwareCapability(
        name="NVIDIA B200", max_threads_per_block=1024, max_block_dim=1024, max_grid_dim=2 ** 31 - 1,
        smem_bytes=232448, smem_bytes_total=233472, supports_fp16=True, supports_bf16=True,
        supports_fp8=True, supports_fp4=True, supports_tf32=True, supports_tensor_core=True,
        supports_winograd=True, max_shared_memory_per_block=232448, compute_capability=(10, 0),
        source="static", verified=False)


def make_strategy(profile: str):
    if profile not in PROFILES:
        raise ValueError(f"unknown plan precision profile {profile!r}; expected one of {PROFILES}")
    from c32.kernel_spec import PrecisionProfile
    from c32.strategy import ExecutionMode, Strategy

    class B200Strategy(Strategy):
        def select_precision(self, node, graph):
            if profile != "fp32" and node.op_type in TENSOR_CORE_OPS:
                return PrecisionProfile(compute_dtype=profile, accumulator_dtype="fp32", input_dtype=profile,
                                        weight_dtype=profile, output_dtype=profile)
            return super().select_precision(node, graph)

    return B200Strategy(hardware=b200_hardware(), mode=ExecutionMode.FULL_FP32)


def build_plan(graph: Any, batch_size: int, profile: str = "bf16"):
    """C3.4 plan of ``graph`` (reference IR, after the C3.3 passes) with the
    B200 precision profile on the tensor-core nodes."""
    from c34.scheduler import ExecutionScheduler

    class B200Scheduler(ExecutionScheduler):
        def __init__(self, *a, **k):
            super().__init__(*a, **k)
            self._strategy = make_strategy(profile)

    plan = B200Scheduler(graph, batch_size=batch_size).build()
    issues = plan.validate()
    if issues:
        raise RuntimeError(f"C3.4 plan failed validation: {issues[:5]}")
    return plan
