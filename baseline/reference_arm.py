"""Runs the UNMODIFIED reference (installed into baseline/_ref) through its own public
API for bench.py's workload shape. Filled in below; until the vLLM path is verified
on a GPU box it reports why it cannot run."""
import json
import os
import sys


def run(args) -> None:
    raise RuntimeError("reference vLLM+AMFKVConnector arm not wired yet")
