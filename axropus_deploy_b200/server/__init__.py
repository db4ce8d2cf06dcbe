from .metrics import MetricRegistry
from .service import EngineService

__all__ = ["MetricRegistry", "EngineService"]
