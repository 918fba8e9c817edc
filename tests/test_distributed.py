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


def test_gloo_data_parallel_groups_match_plain_ranks(tmp_path):
    """dp=2 on 4 ranks (groups {0,1}, {2,3}) gives the same banks as 2 plain ranks: the
    replicas train identical copies and only each group's first member reduces."""
    plain = _launch(tmp_path, "cpu", 2, 29617)
    dp = _launch(tmp_path, "cpu_dp2", 4, 29619)
    for o in dp:
        assert o["consistent"] and o["ckpt_same"] and o["resumed"]
    assert set(dp[0]["losses"][0]) == set(dp[1]["losses"][0]) == {(0, 0), (0, 1)}
    assert set(dp[2]["losses"][0]) == {(1, 0), (1, 1)}
    for r, p in ((0, 0), (1, 0), (2, 1), (3, 1)):
        assert dp[r]["losses"] == plain[p]["losses"]
        for k in plain[p]["bank"]:
            for n in plain[p]["bank"][k]:
                assert torch.equal(dp[r]["bank"][k][n], plain[p]["bank"][k][n]), (r, k, n)


@pytest.mark.gpu
@pytest.mark.multigpu
def test_nvlink_data_parallel_matches_one_rank_per_path_group(tmp_path):
    """Fused executor with every path split over 2 GPUs (peer-memory gradient
    reduce-scatter, sharded AdamW, fused all-gather) against the same four paths on ONE
    GPU (one group = one rank: same placement, same batch generator): same losses and
    banks up to float summation order."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    dp = _launch(tmp_path, "nvlink_dp2", 2, 29621)
    one = _launch(tmp_path, "nccl", 1, 29623)[0]
    for o in dp:
        assert o["consistent"] and o["ckpt_same"] and o["resumed"]
    # both members hold all four paths
    assert set(dp[0]["losses"][0]) == set(dp[1]["losses"][0]) == {(0, 0), (0, 1), (1, 0), (1, 1)}
    for rnd, (a, b) in enumerate(zip(dp[0]["losses"], one["losses"])):
        for path, loss in a.items():
            assert abs(loss - b[path]) < 5e-3 * abs(b[path]), (rnd, path, loss, b[path])
    for k in dp[0]["bank"]:
        for n in dp[0]["bank"][k]:
            assert torch.allclose(dp[0]["bank"][k][n], one["bank"][k][n], atol=2e-3, rtol=2e-2), (k, n)
            assert torch.equal(dp[0]["bank"][k][n], dp[1]["bank"][k][n]), (k, n)


@pytest.mark.gpu
@pytest.mark.multigpu
def test_nvlink_data_parallel_8bit_adam_matches_one_rank(tmp_path):
    """The same with blockwise 8-bit Adam: the shard owner requantises its 256-element
    blocks and stores moments, scales and weights into both members."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    dp = _launch(tmp_path, "nvlink_dp2_8bit", 2, 29625)
    one = _launch(tmp_path, "nccl_8bit", 1, 29627)[0]
    for o in dp:
        assert o["consistent"] and o["resumed"]
    for rnd, (a, b) in enumerate(zip(dp[0]["losses"], one["losses"])):
        for path, loss in a.items():
            assert abs(loss - b[path]) < 1e-2 * abs(b[path]), (rnd, path, loss, b[path])
    for k in dp[0]["bank"]:
        for n in dp[0]["bank"][k]:
            assert torch.allclose(dp[0]["bank"][k][n], one["bank"][k][n], atol=5e-3, rtol=5e-2), (k, n)
            assert torch.equal(dp[0]["bank"][k][n], dp[1]["bank"][k][n]), (k, n)


@pytest.mark.gpu
@pytest.mark.multigpu
def test_nvlink_outer_step_matches_nccl(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    nv = _launch(tmp_path, "nvlink", 2, 29613)
    nc = _launch(tmp_path, "nccl", 2, 29615)
    for a, b in zip(nv, nc):
        assert a["consistent"] and b["consistent"]
        assert a["gather_same"]  # NVLink pull of the full bank == per-parameter broadcast
        assert a["ckpt_same"] and a["resumed"]
        assert a["losses"] == b["losses"]
        for k in a["bank"]:
            for n in a["bank"][k]:
                assert torch.allclose(a["bank"][k][n], b["bank"][k][n], atol=1e-6, rtol=0), (k, n)


@pytest.mark.gpu
@pytest.mark.multigpu
def test_nvlink_int4_outer_step_tracks_uncompressed(tmp_path):
    """int4 codes with error feedback in the NVLink outer step: every sharer ends with the
    same global, round-0 losses are unchanged, and the total update of every shared
    module stays close to the uncompressed run's."""
    from opendipaco_b200.topology import is_private_key

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    q4 = _launch(tmp_path, "nvlink_q4", 2, 29627)
    nv = _launch(tmp_path, "nvlink", 2, 29629)
    for a, b in zip(q4, nv):
        assert a["consistent"] and a["ckpt_same"] and a["resumed"]
        assert a["losses"][0] == b["losses"][0]
        for k in a["bank"]:
            if is_private_key(k):
                continue
            ua = torch.cat([(a["bank"][k][n] - a["init"][k][n]).float().reshape(-1) for n in a["bank"][k]])
            ub = torch.cat([(b["bank"][k][n] - b["init"][k][n]).float().reshape(-1) for n in b["bank"][k]])
            rel = ((ua - ub).norm() / ub.norm().clamp_min(1e-12)).item()
            assert rel < 0.25, (k, rel)


@pytest.mark.gpu
@pytest.mark.multigpu
def test_nvlink_topk_outer_step_stays_consistent(tmp_path):
    """Top-k (5% per 4096-element block) pairs with error feedback in the NVLink outer
    step: sharers stay identical, checkpoints round-trip, round-0 losses are unchanged and
    the shared modules move in the direction of the uncompressed update."""
    from opendipaco_b200.topology import is_private_key

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    sp = _launch(tmp_path, "nvlink_topk", 2, 29631)
    nv = _launch(tmp_path, "nvlink", 2, 29633)
    for a, b in zip(sp, nv):
        assert a["consistent"] and a["ckpt_same"] and a["resumed"]
        assert a["losses"][0] == b["losses"][0]
        for k in a["bank"]:
            if is_private_key(k):
                continue
            ua = torch.cat([(a["bank"][k][n] - a["init"][k][n]).float().reshape(-1) for n in a["bank"][k]])
            ub = torch.cat([(b["bank"][k][n] - b["init"][k][n]).float().reshape(-1) for n in b["bank"][k]])
            cos = torch.nn.functional.cosine_similarity(ua, ub, dim=0).item()
            assert cos > 0.3, (k, cos)
