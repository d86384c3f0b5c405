"""bench.py's output contract and multi-rank plumbing, on the CPU.

The reference arm (the oracle port of the reference's CPU computation) runs here,
so its JSON line can be checked end to end, once directly and once under torchrun
with two ranks (rank 0 alone prints; the other rank exits 0 without work). The
gloo control plane of the GPU arm (barrier, max over ranks, host-object exchange)
is checked with two spawned ranks.
"""
import json
import multiprocessing as mp
import os
from pathlib import Path
import subprocess
import sys

ROOT = Path(__file__).resolve().parents[1]
REFERENCE_ARGS = ["--impl", "reference", "--workload", "add", "--steps", "1", "--warmup", "1"]


def check_reference_line(line, n_gpus):
    assert line["impl"] == "reference" and line["n_gpus"] == n_gpus
    assert line["unit"] == "GB/s" and line["value"] > 0 and line["higher_is_better"] is True
    base = line["cpu_baseline"]
    assert base["kind"] == "port" and base["cores"] >= 1 and base["value"] == line["value"] and base["sample"]
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    sys.path.insert(0, str(ROOT))
    import bench
    metric, unit, scaling, config = bench.describe("add", n_gpus, 0)
    assert (line["metric"], line["unit"], line["scaling"], line["config"]) == (metric, unit, scaling, config)


def test_cpu_baseline_has_all_core_and_single_thread_legs():
    sys.path.insert(0, str(ROOT))
    import bench
    base = bench.cpu_baseline("add", budget=0.2)
    assert base["value"] > 0 and base["single_thread"]["value"] > 0 and base["single_thread"]["cores"] == 1
    assert base["nproc"] >= 1 and "cpu_model" in base


def test_reference_arm_prints_one_line():
    out = subprocess.run([sys.executable, "bench.py", *REFERENCE_ARGS], cwd=ROOT, capture_output=True, text=True,
                         timeout=300)
    assert out.returncode == 0, out.stderr
    lines = [l for l in out.stdout.splitlines() if l.strip()]
    assert len(lines) == 1
    check_reference_line(json.loads(lines[0]), 1)


def test_reference_arm_under_torchrun_rank0_only():
    out = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
                          "--master-addr", "127.0.0.1", "--master-port", "29671", "bench.py", "--gpus", "2",
                          *REFERENCE_ARGS], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr
    lines = [l for l in out.stdout.splitlines() if l.strip().startswith("{")]
    assert len(lines) == 1
    check_reference_line(json.loads(lines[0]), 2)


def _rank(rank, results):
    os.environ.update({"RANK": str(rank), "LOCAL_RANK": str(rank), "WORLD_SIZE": "2", "MASTER_ADDR": "127.0.0.1",
                       "MASTER_PORT": "29672"})
    sys.path.insert(0, str(ROOT))
    import bench
    group = bench.Group(2)
    try:
        group.barrier()
        results.put((rank, group.max(10.0 + rank), group.exchange({"rank": rank})))
    finally:
        group.close()


def test_group_control_plane_over_gloo():
    spawn = mp.get_context("spawn")
    results = spawn.Queue()
    procs = [spawn.Process(target=_rank, args=(r, results)) for r in range(2)]
    for proc in procs:
        proc.start()
    got = dict((r, (m, x)) for r, m, x in (results.get(timeout=120) for _ in range(2)))
    for proc in procs:
        proc.join(timeout=60)
        assert proc.exitcode == 0
    for rank in range(2):
        assert got[rank] == (11.0, [{"rank": 0}, {"rank": 1}])


def test_dominant_entries_name_commands_the_library_records():
    # The roofline's bound follows the variant recorded for the workload's dominant
    # command; a name that no command carries would silently pick the wrong bound.
    sys.path.insert(0, str(ROOT))
    import bench
    # provider commands are named in the runtime, array kernels in the module builder
    files = list((ROOT / "paralyn_b200" / "csrc" / "runtime").glob("*.cpp")) + [ROOT / "paralyn_b200" / "prk.py"]
    sources = "".join(p.read_text() for p in files)
    for workload, entries in bench.DOMINANT_ENTRY.items():
        for entry in (entries,) if isinstance(entries, str) else entries:
            assert f'"{entry}"' in sources, (workload, entry)
