"""Multi-process training: gloo ranks on CPU, and NVLink vs NCCL outer steps on 2 GPUs."""

import os
import subprocess
import sys

import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _launch(tmp_path, mode, nproc, port):
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr=127.0.0.1", f"--master-port={port}",
           os.path.join(HERE, "mp_worker.py"), str(tmp_path), mode]
    env = dict(os.environ, OMP_NUM_THREADS="1")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return [torch.load(tmp_path / f"{mode}_rank{i}.pt", weights_only=False) for i in range(nproc)]


def test_gloo_two_ranks_consistent_and_resumable(tmp_path):
    outs = _launch(tmp_path, "cpu", 2, 29611)
    for o in outs:
        assert o["consistent"] and o["ckpt_same"] and o["resumed"]
    # rank 0 owns paths 0,1 ; rank 1 owns 2,3
    assert set(outs[0]["losses"][0]) == {(0, 0), (0, 1)}
    assert set(outs[1]["losses"][0]) == {(1, 0), (1, 1)}


@pytest.mark.gpu
@pytest.mark.multigpu
def test_nvlink_outer_step_matches_nccl(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    nv = _launch(tmp_path, "nvlink", 2, 29613)
    nc = _launch(tmp_path, "nccl", 2, 29615)
    for a, b in zip(nv, nc):
        assert a["consistent"] and b["consistent"]
        assert a["ckpt_same"] and a["resumed"]
        assert a["losses"] == b["losses"]
        for k in a["bank"]:
            for n in a["bank"][k]:
                assert torch.allclose(a["bank"][k][n], b["bank"][k][n], atol=1e-6, rtol=0), (k, n)
