"""bench.py host logic on CPU: the two arms describe the same workload, the
roofline denominators follow the measured peaks (or the stated fallback), and
the reference arm prints its line on the headline's metric and config."""

import importlib.util
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_headline_config_is_the_same_at_every_call():
    b = _bench()
    assert b.headline_config() == b.headline_config()
    cfg = b.headline_config()
    assert (cfg["M"], cfg["N"], cfg["K"]) == (16384, 16384, 16384)
    assert cfg["products_per_step"] == b.HEAD_PRODUCTS


def test_peaks_int8_denominators_are_twice_bf16(tmp_path, monkeypatch):
    b = _bench()
    pk = b._peaks()
    assert pk["i8_tops"] == 2 * pk["bf16_tflops"]
    assert pk["i8_tops_sustained"] == 2 * pk["bf16_tflops_sustained"]
    monkeypatch.setattr(b, "ROOT", str(tmp_path))  # no peaks file: the stated fallback
    fb = b._peaks()
    assert fb["source"] == "fallback" and fb["hbm_gbs"] == 6650.0 and fb["bf16_tflops"] == 1590.0


def test_reference_arm_prints_the_headline_line():
    env = dict(os.environ, OMP_NUM_THREADS="4")
    res = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1"], capture_output=True, text=True, timeout=600, env=env, cwd=ROOT)
    assert res.returncode == 0, res.stderr[-2000:]
    line = json.loads(res.stdout.strip().splitlines()[-1])
    b = _bench()
    assert line["impl"] == "reference" and line["metric"] == b.METRIC and line["unit"] == "TOPS"
    assert line["config"] == b.headline_config()
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["cpu_baseline"]["kind"] == "port"
    assert line["value"] > 0
