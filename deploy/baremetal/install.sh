#!/usr/bin/env bash
# Install the control-plane binaries, units and configuration on one machine.
#   sudo ./install.sh coord|node      (a node also gets the store)
set -euo pipefail
role=${1:?usage: install.sh coord|node}
here=$(cd "$(dirname "$0")" && pwd)
repo=$(cd "$here/../.." && pwd)
make -C "$repo/cpp" -j"$(nproc)"
getent group everserve >/dev/null || groupadd --system --gid 64000 everserve
id everserve >/dev/null 2>&1 || useradd --system --gid everserve --home /var/lib/everserve --shell /usr/sbin/nologin everserve
install -m 0755 "$repo"/cpp/bin/everserve-{coord,node,store,ctl} /usr/local/bin/
install -d -m 0750 -o everserve -g everserve /etc/everserve
install -m 0644 "$here/everserve.tmpfiles.conf" /etc/tmpfiles.d/everserve.conf
systemd-tmpfiles --create /etc/tmpfiles.d/everserve.conf
if [ "$role" = coord ]; then
  [ -f /etc/everserve/coord.env ] || install -m 0640 "$here/coord.env.example" /etc/everserve/coord.env
  install -m 0644 "$here/everserve-coord.service" /etc/systemd/system/
  systemctl daemon-reload && systemctl enable --now everserve-coord
else
  [ -f /etc/everserve/node.env ] || install -m 0640 "$here/node.env.example" /etc/everserve/node.env
  [ -f /etc/everserve/store.env ] || install -m 0640 "$here/store.env.example" /etc/everserve/store.env
  install -m 0644 "$here/everserve-store.service" "$here/everserve-node.service" /etc/systemd/system/
  systemctl daemon-reload && systemctl enable --now everserve-store everserve-node
fi
