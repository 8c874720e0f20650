"""bench.py's multi-rank plumbing on CPU: two gloo ranks, each standing in
for one GPU replica, agree on the slowest rank's time and the whole-job rate
(no collective on the data path)."""
import os
import socket
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

WORKER = r"""
import os, sys, time
sys.path.insert(0, %r)
import bench
r = bench.Ranks("gloo")
r.barrier()
# rank k "takes" (k + 1) * 10 ms for its steps
t = r.max((r.rank + 1) * 0.010)
rate = bench.aggregate_rate(r.world, 512, 20, t)
r.close()
print("RANK", r.rank, r.world, t, rate, flush=True)
"""


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_two_gloo_ranks_agree_on_max_and_rate():
    port = str(_free_port())
    procs = []
    for rank in range(2):
        env = dict(os.environ, RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE="2",
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=port)
        procs.append(subprocess.Popen([sys.executable, "-c", WORKER % ROOT], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True))
    outs = [p.communicate(timeout=120) for p in procs]
    for p, (o, e) in zip(procs, outs):
        assert p.returncode == 0, e
    lines = [next(l for l in o.splitlines() if l.startswith("RANK")).split() for o, _ in outs]
    for l in lines:
        assert int(l[2]) == 2
        assert abs(float(l[3]) - 0.020) < 1e-12          # the slowest rank's time
        assert abs(float(l[4]) - 2 * 512 * 20 / 0.020) < 1e-6


def test_single_process_needs_no_process_group():
    sys.path.insert(0, ROOT)
    import bench

    env = {k: os.environ.pop(k) for k in ("WORLD_SIZE", "RANK", "LOCAL_RANK") if k in os.environ}
    try:
        r = bench.Ranks("gloo")
        assert r.world == 1 and r.pg is None
        assert r.max(3.5) == 3.5
        r.barrier()
        r.close()
        assert bench.aggregate_rate(1, 512, 10, 2.0) == 2560.0
    finally:
        os.environ.update(env)


def test_reference_arm_prints_one_json_line():
    """bench.py --impl reference (the CPU arm the driver runs next to the
    GPU arm) prints one JSON line with the GPU arm's metric and unit."""
    import json
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, os.path.join(root, "bench.py"), "--impl", "reference",
                        "--workload", "b9c64x6_bs16", "--steps", "2", "--warmup", "3"],
                       capture_output=True, text=True, timeout=600, cwd=root)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "positions/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["e2e"]["value"] == line["value"]
