"""bench.py's N > 1 host logic as two gloo ranks on CPU: barrier, max over
ranks, per-rank stream seeds and the whole-job rate. The data path has no
collective (each GPU runs independent streams), so this is all the multi-GPU
logic there is."""
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _clean_env():
    env = dict(os.environ)
    for k in ("RANK", "LOCAL_RANK", "WORLD_SIZE", "MASTER_ADDR", "MASTER_PORT"):
        env.pop(k, None)
    env["CUDA_VISIBLE_DEVICES"] = ""
    return env


def test_two_ranks_gloo():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(ROOT / "tests" / "multi_rank_worker.py")]
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=240, env=_clean_env(), cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout  # rank 0 alone prints
    rec = json.loads(lines[0])
    assert rec["world"] == 2
    assert rec["slowest"] == 1.5  # rank 1's time, seen by rank 0
    seeds = [tuple(x) for per_rank in rec["seeds"] for x in per_rank]
    assert len(seeds) == 8 and len(set(s[0] for s in seeds)) == 8 and len(set(s[1] for s in seeds)) == 8
    assert abs(rec["rate"] - 2 * 4 * 5 / 1.5) < 1e-9


def test_reference_arm_other_ranks_exit_without_work():
    env = _clean_env()
    env.update({"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"})
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--gpus", "2"],
                         capture_output=True, text=True, timeout=120, env=env, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    assert out.stdout.strip() == ""


def test_single_rank_helpers():
    sys.path.insert(0, str(ROOT))
    import bench
    assert bench.stream_seeds(0, 2) == [(1000, 0), (1001, 1)]
    assert bench.stream_seeds(3, 2) == [(1006, 6), (1007, 7)]
    assert bench.job_rate(8, 16, 20, 2.0) == 8 * 16 * 20 / 2.0
    # bandwidth is per GPU: the whole-job rate of 2 GPUs counts each GPU's share once
    gbs, frac = bench.gpu_bandwidth(2400.0, 2, 4.6e9, 6546.2)
    assert abs(gbs - 1200.0 * 4.6) < 1e-6 and abs(frac - 1200.0 * 4.6 / 6546.2) < 1e-9
    assert bench.gpu_bandwidth(1200.0, 1, 4.6e9, 6546.2) == (gbs, frac)
