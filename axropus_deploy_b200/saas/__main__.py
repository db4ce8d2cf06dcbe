"""``python -m axropus_deploy_b200.saas --port 8080 --db backend.sqlite --upstream http://node:8000``"""
import argparse

import uvicorn

from .app import create_app
from .store import Store


def main() -> None:
    ap = argparse.ArgumentParser(description="axropus-deploy-b200 hosted backend")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8080)
    ap.add_argument("--db", default="axropus_backend.sqlite")
    ap.add_argument("--upstream", default="", help="serving node used when a key's owner has no active deployment")
    ap.add_argument("--bench-dir", default=None, help="directory of benchmark JSON lines")
    ap.add_argument("--public-url", default=None, help="this backend's URL as deployed nodes reach it (starts their agent)")
    a = ap.parse_args()
    uvicorn.run(create_app(Store(a.db), default_upstream=a.upstream, bench_dir=a.bench_dir, backend_url=a.public_url), host=a.host, port=a.port)


if __name__ == "__main__":
    main()
