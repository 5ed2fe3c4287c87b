"""bench.py's reference arm on CPU: one JSON line with the keys the driver reads
(the GPU arm prints the same keys plus roofline, e2e and clocks; it needs a B200)."""

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference",
                          "--steps", "2", "--warmup", "1", "--cpu-seconds", "0.5"],
                         capture_output=True, text=True, timeout=600, check=True).stdout
    lines = [line for line in out.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["steps"] == 2 and d["warmup"] == 1
    assert d["value"] > 0 and d["unit"] == "params/s" and d["higher_is_better"] is True
    installed = (ROOT / "baseline" / "_ref" / "sr_states").is_dir()
    assert d["cpu_baseline"]["kind"] == ("reference" if installed else "port")
    assert d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert "workload" in d["config"]


def _bench():
    import importlib.util

    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module


def test_sample_windows_cover_shard_boundaries_embeddings_and_norms():
    bench = _bench()
    from sr_states.distributed import shard_sizes
    from sr_states.shapes import llama3_8b

    names = [n for n, _ in llama3_8b()]
    shapes = [s for _, s in llama3_8b()]
    total = 8_030_261_248
    for world in (1, 2, 8):
        shard = shard_sizes(total, world)
        windows, offsets = bench.sample_windows(names, shapes, world, shard)
        assert all(a < b for a, b in windows)
        assert all(b1 < a2 for (_, b1), (a2, _) in zip(windows, windows[1:]))  # merged
        covered = lambda x: any(a <= x < b for a, b in windows)  # noqa: E731
        for k in range(1, world):
            assert covered(k * shard - 1) and covered(k * shard)
        for name in ("embed_tokens", "lm_head"):
            start, n = offsets[name]
            assert covered(start) and covered(start + n - 1)
        for name in ("layers.0.input_layernorm", "norm"):
            start, n = offsets[name]
            assert all(covered(start + i) for i in (0, n // 2, n - 1))
