"""Cluster control plane: the AMF coordinator (global prefix index across nodes) and its
fail-open client, the request router with AMF locality and transfer-vs-recompute
costing, durable work queues, the job ledger, per-GPU workers with lane scheduling,
backend adapters, the HTTP gateway, node / worker registries with node-to-node snapshot
transfer, savings accounting, runtime governance and the Dynamo-style integration
components. ``python -m axropus_deploy_b200.cluster`` runs a node, the coordinator or
the admin commands."""
from .coordinator import AmfCoordinator, CoordinatorClient, serve_coordinator
from .ledger import SqliteLedger
from .queues import InProcQueue, SqliteQueue
from .router import ClusterRouter, Route, WorkerInfo

__all__ = ["AmfCoordinator", "CoordinatorClient", "serve_coordinator", "InProcQueue", "SqliteQueue",
           "ClusterRouter", "Route", "WorkerInfo", "SqliteLedger"]
