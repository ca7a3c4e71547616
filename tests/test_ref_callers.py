"""The reference's own callers on this library.

1. ``NesleVecEnv`` (the reference's ``src/nesle/env.py``, CUDA backend, RAM
   observations, auto-reset and truncation).  ``tests/golden/make_ref_callers.py``
   ran the reference's unmodified VecEnv over the reference's batched semantics
   and recorded every call it made to ``nesle._cuda_core.CudaBatch`` with the
   arrays it passed and a digest of every array it got back.  Here the same
   calls, in the same order, go to ``nesle_b200._cuda_core.CudaBatch`` on the GPU
   and must return the same bytes: the reference VecEnv, bound to this module,
   takes exactly the path it takes on its own (the recording needs the
   reference tree; the fixture travels).
2. The rollout loop of the reference's ``native_ppo.py`` (``:471-517``): masks
   on the device, ``step_device(auto_reset=False, synchronize=True)``, done
   masks copied to the host for ``reset_envs``, then ``ram_device()``, all read
   through DLPack -- run in lockstep on this library and on the reference's own
   CUDA module (``oracle/_ref/cuda``, compiled unchanged) on the same GPU.
"""
from __future__ import annotations

import hashlib
import importlib.util
from pathlib import Path

import numpy as np
import pytest

import kat_roms

ROOT = Path(__file__).resolve().parents[1]
FIXTURE = ROOT / "tests" / "golden" / "ref_callers.npz"
REF_DIR = ROOT / "oracle" / "_ref" / "cuda"
OUTPUT_KEYS = {"reset": ("frames",), "ram": ("ram",), "render": ("frames",), "reset_envs": ()}


@pytest.fixture()
def _cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nesle_b200 import build

    build.build()


def digest(a) -> bytes:
    a = np.ascontiguousarray(np.asarray(a))
    return hashlib.sha256(a.dtype.str.encode() + str(a.shape).encode() + a.tobytes()).digest()


class CheckerBatch:
    """The binding's host CudaBatch methods over the CPU checker (oracle/), for the CPU replay."""

    name = "cuda-console"

    def __init__(self, n, frameskip, rom, snaps, env_to_level):
        from oracle import Oracle

        self._o = Oracle(n, frameskip, rom, snaps, env_to_level=env_to_level)

    def reset(self):
        self._o.reset()
        return self._o.render()["rgb"]

    def ram(self):
        return self._o.get("ram")

    def render(self):
        return self._o.render()["rgb"]

    def step(self, actions, render_frame=True, copy_obs=True):
        self._o.step(np.asarray(actions, np.uint8), device_api=False, auto_reset=False)
        out = {"obs": self._o.render()["rgb"]} if copy_obs else {}
        out.update(rewards=self._o.get("reward"), dones=self._o.get("done"))
        return out

    def reset_envs(self, mask):
        self._o.reset_envs(np.asarray(mask, np.uint8))


def _replay(make) -> None:
    d = np.load(FIXTURE)
    methods = [str(m) for m in d["methods"]]
    assert methods[0] == "__init__"
    assert bytes(d["__init___rom_sha"][0]) == hashlib.sha256(kat_roms.ENV_TRACE_ROM).digest()
    n, frameskip, levels = (int(v) for v in d["__init___shape"][0])
    snaps = kat_roms.env_trace_snapshots(levels)
    batch = make(n, frameskip, kat_roms.ENV_TRACE_ROM, snaps, d["__init___env_to_level"][0])
    assert batch.name == "cuda-console"
    want = iter(bytes(row) for row in d["out_digests"])
    cursor = {"step": 0, "reset_envs": 0}
    for i, m in enumerate(methods[1:], start=1):
        if m == "step":
            k = cursor["step"]
            render_frame, copy_obs = (bool(v) for v in d["step_flags"][k])
            out = batch.step(d["step_actions"][k], render_frame=render_frame, copy_obs=copy_obs)
            keys = (("obs",) if copy_obs else ()) + ("rewards", "dones")
            got = [out[key] for key in keys]
            cursor["step"] += 1
        elif m == "reset_envs":
            batch.reset_envs(d["reset_envs_mask"][cursor["reset_envs"]])
            cursor["reset_envs"] += 1
            got = []
        else:
            got = [getattr(batch, m)()]
            assert len(got) == len(OUTPUT_KEYS[m])
        for value in got:
            assert digest(value) == next(want), f"call {i} ({m}) returned different bytes"
    assert next(want, None) is None
    assert int(d["dones_seen"]) > 0 and 0 < int(d["reset_envs_mask"].mean() * 100) < 100


@pytest.mark.gpu
def test_reference_vecenv_call_trace_replays_bit_exact(_cuda):
    from nesle_b200._cuda_core import CudaBatch

    _replay(lambda n, fs, rom, snaps, e2l: CudaBatch(n, fs, rom, snaps, e2l, device=0))


def test_reference_vecenv_call_trace_replays_on_the_checker():
    """The same replay on the CPU checker: pins the checker to the reference under this call pattern."""
    _replay(CheckerBatch)


@pytest.fixture(scope="module")
def ref_cuda():
    found = sorted(REF_DIR.glob("_cuda_core*.so"))
    if not found:
        pytest.skip("reference CUDA binding not built")
    spec = importlib.util.spec_from_file_location("_cuda_core", found[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.gpu
def test_native_ppo_rollout_loop_matches_reference_module(_cuda, ref_cuda):
    """Ten iterations of 16 env-steps of the native_ppo rollout pattern."""
    import torch
    from torch.utils.dlpack import from_dlpack

    from nesle_b200._cuda_core import CudaBatch

    n = 64
    snaps = kat_roms.env_trace_snapshots(8)
    e2l = (np.arange(n) % 8).astype(np.uint8)
    ours = CudaBatch(n, 4, kat_roms.ENV_TRACE_ROM, snaps, e2l, device=0)
    theirs = ref_cuda.CudaBatch(n, 4, kat_roms.ENV_TRACE_ROM, list(snaps), e2l)
    for b in (ours, theirs):
        assert str(b.name) == "cuda-console" and hasattr(b, "step_device") and hasattr(b, "ram_device")
    obs = {id(b): from_dlpack(b.reset_device()).clone() for b in (ours, theirs)}
    np.testing.assert_array_equal(obs[id(ours)].cpu().numpy(), obs[id(theirs)].cpu().numpy())
    table = torch.tensor([0x00, 0x80, 0x81, 0x82, 0x83, 0x01, 0x40], dtype=torch.uint8, device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(7)
    resets = 0
    for it in range(10):
        for step in range(16):
            action = torch.randint(0, 7, (n,), generator=gen, device="cuda")
            masks = table[action].contiguous()
            got = []
            for b in (ours, theirs):
                out = b.step_device(masks, auto_reset=False, synchronize=True)
                done = from_dlpack(out["dones"]).bool()
                ram = from_dlpack(out["ram"]).clone()
                reward = from_dlpack(out["rewards"]).clone()
                if bool(done.any().item()):
                    b.reset_envs(done.to(torch.uint8).cpu().numpy())
                    ram = from_dlpack(b.ram_device()).clone()
                got.append((done.cpu().numpy(), reward.cpu().numpy(), ram.cpu().numpy()))
            for name, x, y in zip(("dones", "rewards", "ram"), got[0], got[1]):
                np.testing.assert_array_equal(x, y, err_msg=f"{name} at iteration {it} step {step}")
            resets += int(got[0][0].sum())
    assert 0 < resets < 10 * 16 * n
