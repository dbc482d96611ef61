# Expert-parallel helpers (names of prism_infer/engine/parallel/__init__.py).
from prism_infer_b200.engine.parallel.expert_parallel import (
    ExpertParallelMoE,
    build_dispatch_plan,
    combine_weighted_sum,
    expert_rank,
    get_expert_parallel_size,
    set_expert_parallel_size,
)

__all__ = [
    "ExpertParallelMoE",
    "build_dispatch_plan",
    "combine_weighted_sum",
    "expert_rank",
    "get_expert_parallel_size",
    "set_expert_parallel_size",
]
