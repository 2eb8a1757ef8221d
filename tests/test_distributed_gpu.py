"""Key-split long-context forward with the CUDA kernels: single process (the
gathers degenerate to local), and 2 NCCL ranks when 2 GPUs are present, each
rank's output shard checked against the oracle's full-sequence forward."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_context_parallel_single_gpu_matches_order2():
    import poly_attention_b200 as P
    from poly_attention_b200.distributed import context_parallel_order2_fwd, zigzag_shard, zigzag_unshard
    torch.manual_seed(0)
    b, h, n, d = 1, 4, 2048, 64
    ts = [torch.randn(b, h, n, d, device="cuda", dtype=torch.bfloat16) for _ in range(4)]
    ref, _, _ = P.poly_attention_order2(ts[0], ts[1], ts[2], ts[3], causal=True)
    out = context_parallel_order2_fwd(*(zigzag_shard(t, 0, 1) for t in ts))
    out = zigzag_unshard([out], 1)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref.float().cpu().numpy(), atol=2e-2, rtol=1e-2)


WORKER = r'''
import os, sys, numpy as np, torch, torch.distributed as dist
sys.path.insert(0, os.environ["POLY_PKG"])
sys.path.insert(0, os.environ["POLY_ROOT"])
from oracle import poly_oracle as O
from poly_attention_b200.distributed import context_parallel_order2_fwd, zigzag_shard
rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank)
dist.init_process_group("nccl", device_id=torch.device("cuda", rank))
torch.manual_seed(0)
b, h, n, d = 1, 4, 4096, 64
ts = [torch.randn(b, h, n, d, device="cuda", dtype=torch.bfloat16) for _ in range(4)]
out = context_parallel_order2_fwd(*(zigzag_shard(t, rank, world) for t in ts))
a = [t.float().cpu().numpy() for t in ts]
ref, _, _ = O.order2_fwd(a[0], a[1], a[1], a[2], a[3], causal=True)
want = zigzag_shard(torch.from_numpy(ref), rank, world).numpy()
got = out.float().cpu().numpy()
err = float(np.abs(got - want).max())
print("rank", rank, "maxerr", err, flush=True)
dist.destroy_process_group()
np.testing.assert_allclose(got, want, atol=2e-2, rtol=1e-2)
'''


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_context_parallel_two_ranks_nccl(tmp_path):
    script = tmp_path / "cp_worker.py"
    script.write_text(WORKER)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, POLY_PKG=os.path.join(root, "poly-attention_b200"), POLY_ROOT=root, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
                        "--master-addr=127.0.0.1", f"--master-port={port}", str(script)],
                       env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
