"""bench.py's reference arm (the reference's own CPU attention, timed on the host cores) prints the
contract's JSON line.  CPU only: the arm runs the reference build in oracle/_ref on full decode steps
of the 32K-context workload (36 layers, 9.66 GB of fp32 cache in host memory), on every host core
whatever OMP_NUM_THREADS says, with the same `config` as the GPU arm."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_contract_line():
    env = dict(os.environ, RANK="0", OMP_NUM_THREADS="1")  # as torchrun exports it
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "0"], cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["unit"] == "tokens/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["config"]["workload"] == "qwen3_8b_decode_32k"
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["gpu_launches"] == 0
    assert d["steps"] == 1 and abs(d["ms_per_step"] - 1e3 / d["value"]) < 1e-6 * d["ms_per_step"]
    sys.path.insert(0, ROOT)
    import bench
    from ligguf_b200.workloads import QWEN3_DECODE_32K
    assert d["config"] == bench.bench_config(QWEN3_DECODE_32K, 1, "p2p")  # the GPU arm's config
    assert cb["cores"] == min(bench.host_cores(), 32)  # all cores, not OMP_NUM_THREADS=1
    assert "36 layers" in cb["sample"]
