"""Fail-stop recovery on GPUs with NCCL training groups (needs 4 GPUs).

Launches ``bench_recovery.py --small`` on 4 GPUs (TP2 x PP2, bf16, fused TP kernels over
peer memory, NCCL with NVLS disabled): rank 3 is SIGKILLed between steps, the survivors
replan onto 3 GPUs, move the lost state and keep training. No GPU is faulted: the kill
happens on the host at a safe point with nothing in flight.
"""

import json
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_failstop_on_four_gpus():
    if torch.cuda.device_count() < 4:
        pytest.skip("needs four GPUs")
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench_recovery.py"), "--gpus", "4", "--small", "--kills", "3:3",
         "--iterations", "6", "--timeout", "400"],
        capture_output=True, text=True, timeout=600, cwd=ROOT,
    )
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["launcher_rc"] == 0, line
    assert line["launch"]["killed_ranks"] == [3]
    ev = line["events"][0]
    assert ev["recovered"] and ev["plan_version"] == 1


def test_failstop_peer_replica_on_four_gpus():
    """TP1 x PP2 x DP2: the lost stage's state comes from the peer replica over NVLink."""
    if torch.cuda.device_count() < 4:
        pytest.skip("needs four GPUs")
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench_recovery.py"), "--gpus", "4", "--layout", "1,2,2", "--small",
         "--kills", "3:3", "--iterations", "6", "--timeout", "400"],
        capture_output=True, text=True, timeout=600, cwd=ROOT,
    )
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["launcher_rc"] == 0, line
    assert line["launch"]["killed_ranks"] == [3]
    ev = line["events"][0]
    assert ev["recovered"] and ev["plan_version"] == 1
    assert line["steps_seen"][-1] == 6


GPU_CONFIG = dict(
    model_dim=256, num_layers=2, num_heads=2, batch_size=8, micro_batch_size=2, seed=0, tp=2, pp=1, dp=2,
    iterations=7, arch="llama", vocab_size=1024, seq_len=256, ffn_dim=512, dtype="bf16", init_std=0.02,
    sequence_parallel=True, lr=1e-3, beta1=0.9, beta2=0.95, weight_decay=0.1, checkpoint_every=1,
)


@pytest.mark.parametrize("hetero", ["nccl", "p2p"])
def test_failstop_resumes_bitwise_like_a_rerun_on_four_gpus(tmp_path, monkeypatch, hetero):
    """TP2 x DP2 with sequence parallelism on four GPUs: the fused TP kernels (AG->GEMM,
    GEMM->RS over peer memory) and the fused DP all-reduce + AdamW run every step. Rank 3
    is SIGKILLed after step 3 (between steps, its GPU idle); the survivors replan onto
    three GPUs (replica 0 keeps TP2, replica 1 continues at TP1), move the lost state and
    resume. Checked: every survivor's installed state equals the checkpoint it resumed
    from, bit for bit (principle A1), and the losses of steps 4-7 equal, bit for bit, an
    uninterrupted run of the new plan started from that checkpoint on three GPUs. The
    replicas' gradients after the failure meet through the logical reduction: bucketed
    NCCL all-reduces (``nccl``) or the peer-memory gather and ordered sum (``p2p``,
    ``RESIHP_P2P_HETERO=1``), in both the failing run and the re-run."""
    if torch.cuda.device_count() < 4:
        pytest.skip("needs four GPUs")
    monkeypatch.setenv("RESIHP_P2P_HETERO", "1" if hetero == "p2p" else "0")
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import dist_entries
    from harness import assert_killed, read_results, run_ranks

    monkeypatch.setenv("NCCL_NVLS_ENABLE", "0")  # no multicast object may be bound to a rank that dies
    kill_after, victim = 3, 3
    fail_dir = tmp_path / "fail"
    fail_dir.mkdir()
    codes = run_ranks(dist_entries.failstop_entry, 4, GPU_CONFIG, {kill_after: victim}, str(fail_dir), True,
                      timeout=500)
    assert_killed(codes, [victim], "gpu failstop")
    survivors = read_results(fail_dir, [0, 1, 2])
    assert all(r["stopped"] is None for r in survivors.values())
    plans = {tuple(r["plans"]) for r in survivors.values()}
    assert len(plans) == 1 and len(next(iter(plans))) == 2
    for r in survivors.values():
        (event,) = r["recoveries"]
        assert event["resumed_from"] == kill_after and event["a1_completed"] == kill_after
        assert event["a1_mismatches"] == [], (r["rank"], event["a1_mismatches"])
        if hetero == "p2p":  # the replicas now differ in layout: the peer-memory gather ran
            assert event["reduction"] == "p2p-hetero", (r["rank"], event["reduction"])
    after = {rank: {int(k): v for k, v in r["losses"].items() if int(k) > kill_after} for rank, r in survivors.items()}
    for rank, losses in after.items():  # every survivor reports its replica's loss of every resumed step
        assert sorted(losses) == list(range(kill_after + 1, GPU_CONFIG["iterations"] + 1)), (rank, losses)

    rerun_dir = tmp_path / "rerun"
    rerun_dir.mkdir()
    anchor = fail_dir / f"anchor_{kill_after}.pt"
    codes = run_ranks(dist_entries.rerun_entry, 3, GPU_CONFIG, [victim], kill_after, str(anchor), str(rerun_dir),
                      True, timeout=500)
    assert set(codes.values()) == {0}
    rerun = {}
    for r in read_results(rerun_dir, [0, 1, 2]).values():
        assert r["plan"] == next(iter(plans))[1]
        rerun[r["rank"]] = {int(k): v for k, v in r["losses"].items()}
    assert rerun == after  # per rank, bitwise: identical floats
