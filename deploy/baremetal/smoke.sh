#!/usr/bin/env bash
# A one-machine control plane in a temporary directory: coordinator, two node daemons and their
# stores. Checks that both nodes link, that a drain reaches the coordinator's event feed, and
# that a daemon's exit is seen as a node loss. Needs only the built binaries (make -C cpp).
set -euo pipefail
repo=$(cd "$(dirname "$0")/../.." && pwd)
bin="$repo/cpp/bin"
dir=$(mktemp -d)
api=127.0.0.1:$((20000 + RANDOM % 20000))
pids=()
cleanup() { for p in "${pids[@]}"; do kill "$p" 2>/dev/null || true; done; rm -rf "$dir"; }
trap cleanup EXIT
echo '{"outcomesInOrder":["OUTCOME_REPLACE"]}' > "$dir/policy.json"
"$bin/everserve-coord" --listen "unix:$dir/coord.sock" --policy "$dir/policy.json" --spec-store "$dir/spec" \
  --lease "$dir/lease" --api-addr "$api" --node-loss-misses 3 > "$dir/coord.log" 2>&1 & pids+=($!)
sleep 0.3
for n in n0 n1; do
  "$bin/everserve-store" --socket "unix:$dir/store-$n.sock" --data-dir "$dir/store-$n" --slots 4096 \
    --budget-bytes 1073741824 > "$dir/store-$n.log" 2>&1 & pids+=($!)
  "$bin/everserve-node" --node "$n" --socket "unix:$dir/$n.sock" --coordinator "unix:$dir/coord.sock" \
    --mirror-socket "unix:$dir/store-$n.sock" --heartbeat-ms 200 > "$dir/$n.log" 2>&1 & pids+=($!)
done
sleep 1
"$bin/everserve-ctl" --api "$api" get nodes | grep -q '"name":"n1"' || { echo "n1 did not link"; exit 1; }
"$bin/everserve-ctl" --api "$api" drain n0 >/dev/null
kill "${pids[4]}"   # n1's daemon
sleep 1.5
events=$("$bin/everserve-ctl" --api "$api" watch --once)
echo "$events"
grep -q "n0 draining" <<<"$events" || { echo "drain not seen"; exit 1; }
grep -q "n1 lost" <<<"$events" || { echo "node loss not seen"; exit 1; }
echo "smoke: ok"
