"""The KV commit path on a B200 with the store's data directory on a disk-backed filesystem.

A rank's gather kernel writes the step's rows straight into the store's staging file when the
file's pages can be pinned (tmpfs, the node's /dev/shm); on other filesystems the host refuses to
pin them and the commit goes through a pinned copy that the sender thread writes into the file.
Both must commit the same rows: this commits from CUDA caches through a store whose data
directory sits under pytest's temporary directory, restores into zeroed caches and compares.
"""

import pytest
import torch

from cpp_bins import Proc, binary, wait_socket
from everserve_b200.state.kvcopy import PagedKV
from everserve_b200.state.mirror import MirrorClient, MirrorCommittedKV

pytestmark = pytest.mark.gpu


def test_commit_restore_from_cuda_caches(tmp_path):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    sock = f"unix:{tmp_path}/store.sock"
    p = Proc([binary("everserve-store"), "--socket", sock, "--data-dir", str(tmp_path / "data"), "--slots", "4096",
              "--budget-bytes", str(1 << 30)])
    try:
        wait_socket(sock)
        kv = PagedKV("heads_blocked", 32, 16, 2, 64)
        g = torch.Generator(device="cuda").manual_seed(1)
        caches = [torch.randn(kv.shape(), device="cuda", generator=g).bfloat16() for _ in range(3)]
        ckv = MirrorCommittedKV(MirrorClient(sock), "eng", 0, caches, kv, store_slots=4096)
        ckv.commit(epoch=1, step=1, counts={"a": 5}, slots=list(range(0, 5)))
        ckv.commit(epoch=1, step=2, counts={"a": 6, "b": 2}, slots=[5, 40, 41])
        ckv.fence(2)
        spare_caches = [torch.zeros_like(c) for c in caches]
        spare = MirrorCommittedKV(MirrorClient(sock), "eng", 1, spare_caches, kv)
        assert spare.restore(0) == {"a": 6, "b": 2}
        heads = torch.arange(kv.heads, device="cuda")
        written = torch.tensor([0, 1, 2, 3, 4, 5, 40, 41], device="cuda")
        for c, s in zip(caches, spare_caches):
            assert torch.equal(kv.rows_of_heads(s, written, heads), kv.rows_of_heads(c, written, heads))
        ckv.close()
        spare.close()
    finally:
        p.stop()
