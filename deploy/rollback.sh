#!/usr/bin/env bash
# Return the compose deployment to the image tag that install.sh replaced last.
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
prev="$(cat "$here/.last_tag" 2>/dev/null || true)"
[ -n "$prev" ] || { echo "no previous tag recorded in deploy/.last_tag" >&2; exit 1; }
docker tag "axropus-b200:$prev" axropus-b200:latest
echo "$prev" > "$here/.current_tag"
docker compose -f "$here/docker-compose.yml" up -d --no-build --force-recreate
echo "rolled back to axropus-b200:$prev"
