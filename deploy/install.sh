#!/usr/bin/env bash
# Build the image and start (or update) the two-node compose deployment.
#   deploy/install.sh [tag]        default tag: the current git commit
# The previous tag is kept in deploy/.last_tag so that deploy/rollback.sh can return to it.
set -euo pipefail
here="$(cd "$(dirname "$0")" && pwd)"
tag="${1:-$(git -C "$here/.." rev-parse --short HEAD)}"
cur="$(cat "$here/.current_tag" 2>/dev/null || true)"
docker build -f "$here/Dockerfile" -t "axropus-b200:$tag" "$here/.."
docker tag "axropus-b200:$tag" axropus-b200:latest
[ -n "$cur" ] && echo "$cur" > "$here/.last_tag"
echo "$tag" > "$here/.current_tag"
docker compose -f "$here/docker-compose.yml" up -d --no-build
echo "deployed axropus-b200:$tag (previous: ${cur:-none})"
