"""Every frame tile of the tensor-core product (16, 32 or 64 frames a CTA;
mma.cu picks one per launch from the shape, TRIT_TC_FRAMES fixes it)
against the CPU oracle: the Q8_0 layers of the Dense tests and the Q8_0,
per-row int8 and ternary mini models through prefill and batched decode
(the tensor-core tests), each run in a process of its own with the tile
fixed, bit for bit as those tests check (src/cpu/int8.rs:560-570)."""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("frames", [16, 32, 64])
def test_frame_tile_matches_oracle(frames):
    env = dict(os.environ, TRIT_TC_FRAMES=str(frames))
    r = subprocess.run(
        [sys.executable, "-m", "pytest", "-x", "-q", "-p", "no:cacheprovider", "tests/test_gpu_tensor_cores.py",
         "tests/test_gpu_dense.py"],
        cwd=ROOT, env=env, capture_output=True, text=True, timeout=1200)
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-2000:]
    assert " passed" in r.stdout and "skipped" not in r.stdout.splitlines()[-1], r.stdout[-1000:]
