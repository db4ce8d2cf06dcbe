"""Hosted backend: accounts, API keys, usage metering and billing, a dashboard, benchmark
data, an OpenAI-compatible inference proxy and SSH deployment of serving nodes. Optional: a
serving node runs without it."""
from .app import create_app
from .store import Store, make_token, read_token

__all__ = ["create_app", "Store", "make_token", "read_token"]
