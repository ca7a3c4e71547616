"""Record how the reference's own VecEnv drives its CUDA module, as a fixture.

Runs the reference's unmodified ``nesle`` package (``src/nesle/env.py``,
imported read-only from the reference tree, no bytecode written there) with
``nesle._cuda_core`` bound to a recording stand-in.  The stand-in implements
the binding's host-side ``CudaBatch`` methods that ``NesleVecEnv`` calls on the
CUDA path (constructor, ``name``, ``reset``, ``ram``, ``step``, ``render``,
``reset_envs``) with the reference's own batched semantics compiled on the CPU
(``oracle/_ref``, kind "B": ``kernels.cu:19-104`` over the ``batch_*.cuh``
headers, the SMB done predicate of the binding).  Every call is stored with its
array arguments and a SHA-256 of every array it returns.

``tests/test_ref_callers.py`` replays the recorded calls on
``nesle_b200._cuda_core.CudaBatch`` on a GPU and requires the same digests:
the reference's VecEnv, running on this library, would see exactly what it
sees on the reference's module.

The workload: ``kat_roms.ENV_TRACE_ROM`` and its 8 level snapshots written to
files (the reference binding has only the SMB done predicate; in this ROM an
env is done when its action holds A for a whole env-step, so auto-reset masks
are partial), 16 envs, ``action_space="simple"``, ``observation_mode="ram"``,
``max_episode_steps=12`` (truncation resets as well), 160 ``step`` calls and
20 ``step_reward`` calls with seeded random action indices, one ``render``.

Usage (needs the reference tree and a built ``oracle/_ref``)::

    python tests/golden/make_ref_callers.py
"""
from __future__ import annotations

import hashlib
import os
import sys
import tempfile
import types
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
# The reference checkout: NESLE_REFERENCE, else a sibling of this repository (as oracle/Makefile).
REF_SRC = Path(os.environ.get("NESLE_REFERENCE", ROOT.parent / "reference")) / "src"
OUT = Path(__file__).with_name("ref_callers.npz")
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))
sys.dont_write_bytecode = True  # nothing is written into the reference tree

import kat_roms  # noqa: E402
from oracle import Reference, build  # noqa: E402

NUM_ENVS, STEPS, REWARD_STEPS, MAX_EPISODE_STEPS = 16, 160, 20, 12


def digest(a) -> bytes:
    """SHA-256 over an array's dtype, shape and bytes (tests/test_ref_callers.py computes the same)."""
    a = np.ascontiguousarray(np.asarray(a))
    return hashlib.sha256(a.dtype.str.encode() + str(a.shape).encode() + a.tobytes()).digest()


class Recorder:
    def __init__(self) -> None:
        self.calls: list[tuple[str, dict, dict]] = []  # (method, array arguments, output digests)

    def add(self, method: str, args: dict, outs: dict) -> None:
        self.calls.append((method, {k: np.asarray(v).copy() for k, v in args.items()},
                           {k: digest(v) for k, v in outs.items()}))


REC = Recorder()


class RecordingCudaBatch:
    """The binding's CudaBatch host methods over the reference's batched semantics on the CPU."""

    def __init__(self, num_envs, frameskip, rom_bytes=None, snapshots=None, env_to_level=None):
        if rom_bytes is None:
            raise ValueError("the recording stand-in needs a ROM")
        snaps = [] if snapshots is None else ([snapshots] if isinstance(snapshots, (bytes, bytearray))
                                              else list(snapshots))
        e2l = None if env_to_level is None else np.asarray(env_to_level, np.uint8)
        self._n = num_envs
        self._ref = Reference("B", num_envs, frameskip, bytes(rom_bytes), [bytes(s) for s in snaps],
                              env_to_level=e2l)
        args = {"rom_sha": np.frombuffer(hashlib.sha256(bytes(rom_bytes)).digest(), np.uint8),
                "shape": np.array([num_envs, frameskip, len(snaps)], np.int64)}
        if e2l is not None:
            args["env_to_level"] = e2l
        REC.add("__init__", args, {})

    @property
    def name(self) -> str:
        return "cuda-console"

    def reset(self):
        self._ref.reset()
        frames = self._ref.render_rgb()
        REC.add("reset", {}, {"frames": frames})
        return frames

    def ram(self):
        out = self._ref.get("ram")
        REC.add("ram", {}, {"ram": out})
        return out

    def step(self, actions, render_frame=True, copy_obs=True):
        a = np.ascontiguousarray(actions, dtype=np.uint8)
        self._ref.step(a, device_api=False, auto_reset=False)
        out = {}
        if copy_obs:
            out["obs"] = self._ref.render_rgb()
        out["rewards"] = self._ref.get("reward")
        out["dones"] = self._ref.get("done")
        REC.add("step", {"actions": a, "flags": np.array([render_frame, copy_obs], np.uint8)}, out)
        return out

    def render(self):
        frames = self._ref.render_rgb()
        REC.add("render", {}, {"frames": frames})
        return frames

    def reset_envs(self, mask):
        m = np.ascontiguousarray(mask, dtype=np.uint8)
        self._ref.reset_envs(m)
        REC.add("reset_envs", {"mask": m}, {})


def main() -> int:
    build()
    if not REF_SRC.exists():
        raise SystemExit("the reference tree is needed to record the fixture")
    sys.path.insert(0, str(REF_SRC))
    import nesle  # the reference package

    fake = types.ModuleType("nesle._cuda_core")
    fake.CudaBatch = RecordingCudaBatch
    sys.modules["nesle._cuda_core"] = fake
    nesle._cuda_core = fake

    with tempfile.TemporaryDirectory() as tmp:
        rom_path = Path(tmp) / "trace.nes"
        rom_path.write_bytes(kat_roms.ENV_TRACE_ROM)
        state_paths = []
        for k, snap in enumerate(kat_roms.env_trace_snapshots()):
            p = Path(tmp) / f"level{k}.fcs"
            p.write_bytes(snap)
            state_paths.append(str(p))
        env = nesle.make_vec(str(rom_path), num_envs=NUM_ENVS, frameskip=4, action_space="simple", backend="cuda",
                             observation_mode="ram", reset_state_paths=state_paths,
                             max_episode_steps=MAX_EPISODE_STEPS, seed=0)
        rng = np.random.default_rng(20261202)
        obs = env.reset()
        env_digests = [digest(obs)]
        dones_seen = 0
        for _ in range(STEPS):
            obs, rew, dones, infos = env.step(rng.integers(0, 7, NUM_ENVS))
            dones_seen += int(np.asarray(dones).sum())
            terminal = [infos[i]["terminal_observation"] for i in range(NUM_ENVS) if "terminal_observation" in infos[i]]
            env_digests.append(hashlib.sha256(digest(obs) + digest(rew) + digest(dones) +
                                              b"".join(digest(t) for t in terminal)).digest())
        for _ in range(REWARD_STEPS):
            rew, dones, infos = env.step_reward(rng.integers(0, 7, NUM_ENVS))
            dones_seen += int(np.asarray(dones).sum())
        env.render()
        env.close()

    # Packed in call order: a method per call, the array arguments of each
    # method stacked in the order of its calls, and the output digests of every
    # call in order (per call, the keys its method returns, in the order above).
    arrays = {"methods": np.array([c[0] for c in REC.calls]), "dones_seen": np.array(dones_seen),
              "env_digests": np.frombuffer(b"".join(env_digests), np.uint8).reshape(-1, 32)}
    packed: dict[str, list] = {}
    digests = []
    for method, args, outs in REC.calls:
        for k, v in args.items():
            packed.setdefault(f"{method}_{k}", []).append(v)
        digests.extend(outs.values())
    for k, v in packed.items():
        arrays[k] = np.stack(v)
    arrays["out_digests"] = np.frombuffer(b"".join(digests), np.uint8).reshape(-1, 32)
    np.savez_compressed(OUT, **arrays)
    kinds = {m: int((arrays["methods"] == m).sum()) for m in set(arrays["methods"].tolist())}
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes): {len(REC.calls)} calls {kinds}, {dones_seen} dones")
    return 0


if __name__ == "__main__":
    sys.exit(main())
