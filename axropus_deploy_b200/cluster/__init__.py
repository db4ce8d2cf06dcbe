"""Cluster control plane: the AMF coordinator (global prefix index across nodes), its
fail-open client, the request router with AMF locality and transfer-vs-recompute
costing, and durable work queues."""
from .coordinator import AmfCoordinator, CoordinatorClient, serve_coordinator
from .queues import InProcQueue, SqliteQueue
from .router import ClusterRouter, Route, WorkerInfo

__all__ = ["AmfCoordinator", "CoordinatorClient", "serve_coordinator", "InProcQueue", "SqliteQueue",
           "ClusterRouter", "Route", "WorkerInfo"]
