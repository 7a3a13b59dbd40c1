from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable


@dataclass(frozen=True)
class MetricDefinition:
    """A named function from a record's raw_metrics to one derived number
    (reference: src/teamredbench/metrics/base.py)."""

    name: str
    description: str
    compute: Callable[[dict[str, Any]], float | None]
