"""The reference's own device path, unchanged, on this library.

oracle/_ref/forward_on_b200 is mini_llama's forward.cpp, model.cpp (weight
upload) and sampler, compiled from the reference sources and linked against
the adapter (mini_llama_b200/adapter: the reference CUDA headers implemented
over the C ABI) instead of the reference CUDA sources.  Its greedy tokens must
equal the reference CPU path's (golden fixtures).  gpu_core_test_b200 is the
reference's own GPU unit test (test/gpu_core_test.cpp) on the same build.
"""
import json
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu
REF = os.path.join(ROOT, "oracle", "_ref")


def run(args, timeout=600):
    exe = os.path.join(REF, args[0])
    if not os.path.exists(exe):
        pytest.fail(f"{exe} missing: build with make -C oracle ref-b200 (needs the reference tree)")
    return subprocess.run([exe] + args[1:], capture_output=True, text=True, timeout=timeout)


def test_reference_gpu_unit_test_passes_on_this_library():
    r = run(["gpu_core_test_b200"])
    assert r.returncode == 0, r.stdout + r.stderr
    assert "PASS gpu-core-test" in r.stdout


@pytest.mark.parametrize("name,fixture,prompt,new", [
    ("tiny", "golden_tiny", 4, 8),
    ("llama2_l2", "golden_llama", 6, 6),
    ("qwen2", "golden_qwen2", 64, 128),
])
def test_unchanged_forward_cpp_greedy_tokens(request, name, fixture, prompt, new):
    golden = request.getfixturevalue(fixture)
    r = run(["forward_on_b200", name, str(prompt), str(new)])
    assert r.returncode == 0, r.stderr
    out = json.loads(r.stdout.strip().splitlines()[-1])
    gen = np.array(out["generated"])
    ref = golden[f"model_{name}_generated"]
    mismatch = np.flatnonzero(gen != ref)
    assert mismatch.size == 0, f"{name}: first mismatching generated token {mismatch[:3]}"
    # top-1 logit of every greedy step against the reference CPU path
    top = golden[f"model_{name}_top_val"].reshape(-1, 8)[prompt - 1:, 0]
    scale = max(1.0, float(np.abs(top).max()))
    assert float(np.abs(np.array(out["top1"]) - top).max()) <= 1e-3 * scale
