"""Host logic of bench.py (CPU): the strong split of config 2's 64 slots over N GPUs, the config
object both arms print, and the reference arm's bounded CPU leg (the reference build's own
full_attention + recurrent_delta_step, one step = every slot once, windows growing by one)."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_slots_split_evenly_and_balanced(world):
    lens = bench.slot_lengths(1000)
    parts = bench.assign_slots(lens, world)
    assert sorted(s for p in parts for s in p) == list(range(len(lens)))
    assert {len(p) for p in parts} == {len(lens) // world}
    loads = [sum(lens[s] for s in p) for p in parts]
    # longest first onto the least-loaded rank: no rank more than one longest window above another
    assert max(loads) - min(loads) <= max(lens)
    if world > 1:
        assert max(loads) / (sum(loads) / world) < 1.05


def test_both_arms_print_the_same_config():
    class A:
        kv_lo, kv_hi = 1024, 32768
    for world in (1, 2, 8):
        c = bench.config2_desc(world, A())
        assert c["global_slots"] == 64 and c["slots_per_gpu"] == 64 // world
        assert json.dumps(c) == json.dumps(bench.config2_desc(world, A()))


def test_reference_cpu_leg_steps_every_slot_with_growth(oracle_lib):
    """The CPU leg in its own process: 3 slots, 2 timed steps after 1 warm-up step."""
    if not oracle_lib.have_ref():
        pytest.skip("reference build not present")
    spec = json.dumps({"task": "decode", "lens": [300, 700, 1500], "steps": 2, "warmup": 1,
                       "budget_s": 30.0, "threads": 2})
    env = dict(os.environ, OMP_NUM_THREADS="2", CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--cpu-json", spec],
                       capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["steps"] == 2 and res["slots"] == 3
    assert res["tok_s"] > 0 and res["seconds"] > 0


def test_reference_recurrent_leg_steps_thirty_layers(oracle_lib):
    """Config 1's CPU leg in its own process: the reference's recurrent_delta_step over the 30
    layers of one slot, 2 timed steps."""
    if not oracle_lib.have_ref():
        pytest.skip("reference build not present")
    spec = json.dumps({"task": "recurrent", "steps": 2, "threads": 2})
    env = dict(os.environ, OMP_NUM_THREADS="2", CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--cpu-json", spec],
                       capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["steps"] == 2 and res["tok_s"] > 0 and res["step_s"] > 0
