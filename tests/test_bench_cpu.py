"""bench.py's reference arm keeps the JSON contract the driver reads (CPU)."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def _run(*args):
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True,
                         text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def test_reference_arm_line():
    d = _run("--impl", "reference", "--config", "c1", "--steps", "2", "--warmup", "1")
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["value"] > 0 and d["steps"] == 2
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["value"] == d["value"] and cb["sample"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0


def test_block_config_reference_arm_is_declared_unavailable():
    d = _run("--impl", "reference", "--config", "c3")
    assert d["impl"] == "reference" and "unavailable" in d


def test_block_cpu_baseline_sample_runs_small():
    sys.path.insert(0, str(ROOT))
    import bench
    steps_per_s, secs = bench.cpu_block_sample(txt_len=8, grid=4, dim=256, heads=2, rank_lora=4)
    assert steps_per_s > 0 and secs > 0


def test_reference_arm_row_sample_counts_its_flops():
    sys.path.insert(0, str(ROOT))
    import numpy as np

    import bench
    from foundry_trainer_b200 import configs
    from oracle import attn_oracle as orc
    pos = configs.positions(8, 4).numpy()  # S = 24
    g = np.random.default_rng(0)
    qn, kn, vn, dn = (g.standard_normal((24, 1, 128)).astype(np.float32) for _ in range(4))
    assert bench._oracle_rows_step(orc, qn, kn, vn, dn, pos, 6) == 14.0 * 6 * 24 * 128


def test_reference_arm_other_ranks_exit_quietly():
    import os
    env = dict(os.environ, RANK="1", WORLD_SIZE="2", LOCAL_RANK="1")
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "1"], capture_output=True, text=True,
                         timeout=600, cwd=ROOT, env=env)
    assert out.returncode == 0, out.stderr[-2000:]
    assert not [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
