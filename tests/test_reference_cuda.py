"""Bit-exactness against the reference's own CUDA kernel on the same B200.

The reference's pybind11 CUDA module (cpp/bindings/cuda_module.cu with
cpp/src/cuda/kernels.cu, compiled unchanged for sm_100a into oracle/_ref/cuda
by `make -C oracle ref-cuda`) and this library step the same ROM, snapshots
and actions with the reference's done predicate (SMB, the only one its kernel
has) through `step_device(auto_reset=True)`; RAM, rewards and dones must agree
after every step, and the rendered RGB frames at the end.  This library's step
runs first each time: the reference kernel executes `trap` on an illegal
opcode, so the reference only runs a step that this library completed without
one.
"""
from __future__ import annotations

import importlib.util
from pathlib import Path

import numpy as np
import pytest

from nesle_b200 import workloads as w

pytestmark = pytest.mark.gpu

REF_DIR = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "cuda"


@pytest.fixture(scope="module")
def ref():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    found = sorted(REF_DIR.glob("_cuda_core*.so"))
    if not found:
        pytest.skip("reference CUDA binding not built")
    spec = importlib.util.spec_from_file_location("_cuda_core", found[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    from nesle_b200 import build

    build.build()
    return mod


def _pair(ref, wl, n):
    from nesle_b200._cuda_core import CudaBatch
    from nesle_b200.native_ppo import batch_snapshot_args

    snap, e2l = batch_snapshot_args(wl, np.arange(n))
    ours = CudaBatch(n, wl.frameskip, wl.rom.image, snap, e2l, device=0, done_mode=w.DONE_SMB)
    if snap is None:
        theirs = ref.CudaBatch(n, wl.frameskip, wl.rom.image)
    elif e2l is None:
        theirs = ref.CudaBatch(n, wl.frameskip, wl.rom.image, snap)
    else:
        theirs = ref.CudaBatch(n, wl.frameskip, wl.rom.image, list(snap), e2l)
    return ours, theirs


def _host(view):
    import torch

    return torch.utils.dlpack.from_dlpack(view).cpu().numpy()


@pytest.mark.parametrize("make,n", [(w.config1, 64), (w.config2, 256), (w.config3, 256), (w.config4, 512)])
def test_step_device_matches_reference_cuda_kernel(ref, make, n):
    import torch

    wl = make()
    ours, theirs = _pair(ref, wl, n)
    env = np.arange(n)
    np.testing.assert_array_equal(_host(ours.reset_device()), _host(theirs.reset_device()))
    resets = 0
    for s in range(6):
        a = torch.from_numpy(wl.actions(env, s)).cuda()
        o = ours.step_device(a, auto_reset=True, synchronize=True)  # raises on an illegal opcode
        t = theirs.step_device(a, auto_reset=True, synchronize=True)
        np.testing.assert_array_equal(_host(o["ram"]), _host(t["ram"]), err_msg=f"ram step {s}")
        np.testing.assert_array_equal(_host(o["rewards"]), _host(t["rewards"]), err_msg=f"rewards step {s}")
        np.testing.assert_array_equal(_host(o["dones"]), _host(t["dones"]), err_msg=f"dones step {s}")
        resets += int(_host(o["dones"]).sum())
    np.testing.assert_array_equal(ours.render(), np.asarray(theirs.render()))
    np.testing.assert_array_equal(ours.oam(), np.asarray(theirs.oam()))
