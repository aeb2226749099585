"""Multi-GPU paths: runs tests/mgpu_worker.py under torchrun, one process per GPU (2, or up
to 8 with CKL_EP_TEST_GPUS), and requires every rank's result file. Attention by KV head
with the fused gather, and one long sequence split by chunks over the GPUs with rank 0's
LSE merge, must equal the single-GPU decode exactly (rank 0 checks); the
expert-parallel MoE layer must match the single-GPU layer and a fp32 reference (within
1e-3 and 1e-2 relative RMS; each rank checks its own tokens). Skipped with fewer than 2
GPUs."""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _ngpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.skipif(_ngpus() < 2, reason="needs 2 GPUs")
def test_head_parallel_attention_and_expert_parallel_moe(tmp_path):
    n = min(_ngpus(), int(os.environ.get("CKL_EP_TEST_GPUS", "2")), 8)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", CKL_EP_RESULT_DIR=str(tmp_path))
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={n}", "--master-addr=127.0.0.1",
           f"--master-port={port}", os.path.join(ROOT, "tests", "mgpu_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    sys.stdout.write(r.stdout[-4000:])
    # the workers' own tracebacks (torchrun's summary alone names no cause)
    tb = [l for l in (r.stdout + r.stderr).splitlines()
          if l.startswith("[rank") or "Error" in l or "assert" in l]
    assert r.returncode == 0, "\n".join(tb[-60:])
    for rank in range(n):
        with open(tmp_path / f"rank{rank}.json") as f:
            res = json.load(f)
        assert [c["case"] for c in res] == ["attn_config1_3chunks", "attn_64x1024_direct",
                                            "attn_B1_seqsplit_8000", "config4_T64_per_rank",
                                            "config4_ragged", "config5_T32"]
        for c in res:
            if "rel_rms_vs_fp32" in c:
                assert c["rel_rms_vs_fp32"] <= 1e-2 and c["rel_rms_vs_single_gpu"] < 1e-3, c
