"""Aggregated configuration (reference config.py:10-17)."""

from __future__ import annotations

from dataclasses import asdict, dataclass, field

from underhfs_b200.compile import CompilePolicy
from underhfs_b200.cuda import RuntimePolicy
from underhfs_b200.distributed import DistributedPolicy


@dataclass
class UnderHFSConfig:
    runtime: RuntimePolicy = field(default_factory=RuntimePolicy)
    compile: CompilePolicy = field(default_factory=CompilePolicy)
    distributed: DistributedPolicy = field(default_factory=DistributedPolicy)

    def to_dict(self) -> dict:
        return asdict(self)
