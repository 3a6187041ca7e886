"""HostGather with the buffer page-locked (the multi-GPU end-to-end path of bench.py): a
device tensor copied asynchronously into this rank's slice lands byte for byte, twice in a row,
and closing the gather unlinks the shared-memory segment.  One rank (a gloo group of one) is
enough to exercise the registration and the asynchronous copy; the gather across ranks is
covered on the CPU in tests/test_shard.py."""
import os
import socket

import pytest

pytestmark = pytest.mark.gpu


def test_host_gather_page_locked_copies_from_the_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import torch.distributed as dist
    from perm_b200.shard import HostGather
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        n = (5 << 20) + 3
        hg = HostGather(torch, dist, [n], 0, 1, register=True)
        assert hg.registered and hg.mine.numel() == n
        name = hg.shm.name
        side = torch.cuda.Stream()
        for seed in (1, 2):
            src = torch.randint(0, 256, (n,), dtype=torch.uint8, device="cuda",
                                generator=torch.Generator(device="cuda").manual_seed(seed))
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                hg.mine.copy_(src, non_blocking=True)
            side.synchronize()
            hg.barrier()
            assert torch.equal(hg.view[:n], src.cpu())
        hg.close()
        assert not os.path.exists(os.path.join("/dev/shm", name.lstrip("/")))
    finally:
        dist.destroy_process_group()
