"""bench.py's contract on a machine without a GPU: the reference arm (the
reference's CPU torch path) prints its JSON line, and the library's own arm
refuses to run rather than fall back to the CPU."""
import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(args, env_extra=None, timeout=600):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, os.path.join(REPO, "bench.py")] + args, cwd=REPO, env=env,
                          capture_output=True, text=True, timeout=timeout)


def test_reference_arm_prints_its_json_line():
    r = _run(["--impl", "reference", "--steps", "1", "--warmup", "0"])
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0 and line["unit"] == "TFLOPS"
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0


def test_library_arm_refuses_without_a_gpu():
    r = _run(["--steps", "1", "--warmup", "0", "--no-cpu-baseline", "--no-e2e", "--no-ep",
              "--no-mixtral"], env_extra={"CUDA_VISIBLE_DEVICES": ""}, timeout=300)
    assert r.returncode != 0
    assert '"value"' not in r.stdout
