"""SB3-style vector environment over the batched core (host VecEnv path).

Restates the CUDA branch of the reference's ``nesle.env.NesleVecEnv``
(src/nesle/env.py:420-757): ``reset``, ``step_async`` / ``step_wait`` /
``step`` with the SB3 auto-reset contract (a done env's pre-reset observation
in ``infos[i]["terminal_observation"]``, the returned observation already from
the new episode), ``step_reward`` for reward-only loops, optional
``max_episode_steps`` truncation and an observation cadence for image modes.

Differences that keep the host path cheap: action indices become joypad masks
with one vectorised lookup; RAM, rewards and dones come back with
non-blocking copies into fresh page-locked buffers and one synchronisation
per step (the reference issues three synchronous copies, env.py:596-647);
after resets only the reset envs' rows are read again.
"""
from __future__ import annotations

from collections.abc import Iterable, Sequence
from typing import Any

import numpy as np

from . import workloads as w


class NesleVecEnv:
    """Vector env of ``num_envs`` consoles on one GPU.

    ``observation_mode``: "ram" (N, 2048), "rgb_array" (N, 240, 256, 3) or
    "gray84" (N, 84, 84).  ``action_masks``: the joypad byte of each discrete
    action (default: the reference's SIMPLE_MOVEMENT table).  ``batch``: an
    existing object with the CudaBatch interface (tests inject one).
    """

    metadata = {"render_modes": ["rgb_array"], "render_fps": 60}

    def __init__(self, rom_bytes: bytes | None, num_envs: int, frameskip: int = 4,
                 action_masks: Sequence[int] = w.SIMPLE_MOVEMENT_MASKS, observation_mode: str = "ram",
                 snapshots: Sequence[bytes] | None = None, env_to_level: Sequence[int] | None = None,
                 max_episode_steps: int = 0, observation_cadence: int = 1, device: int = 0,
                 batch: Any = None, **batch_kw: Any) -> None:
        if num_envs <= 0:
            raise ValueError("num_envs must be positive")
        if frameskip <= 0:
            raise ValueError("frameskip must be positive")
        if observation_cadence <= 0:
            raise ValueError("observation_cadence must be positive")
        if observation_mode not in ("ram", "rgb_array", "gray84"):
            raise ValueError("observation_mode must be 'ram', 'rgb_array' or 'gray84'")
        self.num_envs = num_envs
        self.frameskip = frameskip
        self.observation_mode = observation_mode
        self.observation_cadence = observation_cadence
        self.max_episode_steps = max_episode_steps
        self.action_masks = np.asarray(list(action_masks), dtype=np.uint8)
        if batch is None:
            from ._cuda_core import CudaBatch

            snaps = list(snapshots) if snapshots else []
            if len(snaps) > 1:
                e2l = (np.arange(num_envs) % len(snaps)).astype(np.uint8) if env_to_level is None else \
                    np.asarray(env_to_level, dtype=np.uint8)
                if e2l.shape != (num_envs,):
                    raise ValueError(f"env_to_level shape must be ({num_envs},), got {e2l.shape}")
                batch = CudaBatch(num_envs, frameskip, rom_bytes, snaps, e2l, device=device, **batch_kw)
            else:
                batch = CudaBatch(num_envs, frameskip, rom_bytes, snaps[0] if snaps else None, device=device,
                                  **batch_kw)
        self._batch = batch
        self._torch = None
        if hasattr(batch, "ram_device"):
            try:
                import torch

                if torch.cuda.is_available():
                    self._torch = torch
            except ImportError:  # pragma: no cover
                pass
        self._steps = np.zeros(num_envs, dtype=np.int64)
        self._step_count = 0
        self._obs_cache: np.ndarray | None = None
        self._pending: np.ndarray | None = None
        self.reset_infos: list[dict[str, Any]] = [{} for _ in range(num_envs)]
        self.buf_infos: list[dict[str, Any]] = [{} for _ in range(num_envs)]

    # -- copies ---------------------------------------------------------------
    def _pinned(self, view):
        """Fresh page-locked host array filled from a device view (non-blocking)."""
        torch = self._torch
        src = torch.utils.dlpack.from_dlpack(view)
        dst = torch.empty(src.shape, dtype=src.dtype, pin_memory=True)
        dst.copy_(src, non_blocking=True)
        return dst

    def _step_outputs(self, with_ram: bool) -> tuple[np.ndarray | None, np.ndarray, np.ndarray]:
        """(RAM or None, rewards, dones) of the last host step, one synchronisation."""
        b = self._batch
        if self._torch is None:
            ram = np.asarray(b.ram(), np.uint8) if with_ram else None
            return ram, np.asarray(b.get_field("rewards"), np.float32), np.asarray(b.get_field("done"), bool)
        from . import _lib
        from ._cuda_core import CudaDeviceArrayView

        # step() (not step_device) results: the rewards / done arrays, not last_*
        rew_v = CudaDeviceArrayView(b, b._ptr(_lib.PTR_REWARDS)[0], (self.num_envs,), "<f4")
        done_v = CudaDeviceArrayView(b, b._ptr(_lib.PTR_DONE)[0], (self.num_envs,), "|u1")
        ram = self._pinned(b.ram_device()) if with_ram else None
        rew = self._pinned(rew_v)
        done = self._pinned(done_v)
        self._torch.cuda.current_stream(b.device).synchronize()
        b._raise_on_fault()  # illegal-opcode env faults stay loud
        return (ram.numpy() if ram is not None else None), rew.numpy(), done.numpy().astype(bool)

    def _launch(self, masks: np.ndarray) -> None:
        if self._torch is not None and hasattr(self._batch, "step_launch"):
            self._batch.step_launch(masks)  # results come back through _step_outputs' copies
        else:
            self._batch.step(masks, render_frame=False, copy_obs=False)

    def _frames(self) -> np.ndarray:
        if self.observation_mode == "gray84":
            self._batch.obs_gray84_device(render=True)
            return np.asarray(self._batch.get_field("obs_gray84"), np.uint8)
        return np.asarray(self._batch.render(), np.uint8)

    def _rows(self, idx: np.ndarray) -> np.ndarray:
        """Current observations of envs `idx` only."""
        if self.observation_mode != "ram":
            return self._frames()[idx]
        if self._torch is None:
            return np.asarray(self._batch.ram(), np.uint8)[idx]
        ram = self._torch.utils.dlpack.from_dlpack(self._batch.ram_device())
        sel = ram[self._torch.as_tensor(idx, device=ram.device)]
        return sel.cpu().numpy()

    def _masks(self, actions: Iterable[int]) -> np.ndarray:
        a = np.asarray(actions, dtype=np.int64).ravel()
        if a.shape != (self.num_envs,):
            raise ValueError(f"expected actions with shape ({self.num_envs},), got {a.shape}")
        if (a < 0).any() or (a >= len(self.action_masks)).any():
            raise ValueError("action index out of range")
        return self.action_masks[a]

    def _info(self, **extra: Any) -> dict[str, Any]:
        d = {"backend": str(self._batch.name), "observation_mode": self.observation_mode}
        d.update(extra)
        return d

    # -- VecEnv API -------------------------------------------------------------
    def reset(self) -> np.ndarray:
        self._batch.reset_device()
        self._steps[:] = 0
        self._step_count = 0
        obs = np.asarray(self._batch.ram(), np.uint8) if self.observation_mode == "ram" else self._frames()
        self._obs_cache = None if self.observation_mode == "ram" else obs
        self.reset_infos = [self._info() for _ in range(self.num_envs)]
        return obs

    def step_async(self, actions: Iterable[int]) -> None:
        self._pending = np.asarray(actions, dtype=np.int64).ravel()
        if self._pending.shape != (self.num_envs,):
            raise ValueError(f"expected actions with shape ({self.num_envs},), got {self._pending.shape}")

    def step_wait(self):
        if self._pending is None:
            raise RuntimeError("step_async must be called before step_wait")
        return self.step(self._pending)

    def _done_and_truncation(self, dones: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
        if self.max_episode_steps > 0:
            trunc = self._steps >= self.max_episode_steps
            return dones | trunc, trunc
        return dones, np.zeros(self.num_envs, dtype=bool)

    def step(self, actions: Iterable[int]):
        """SB3 step: (observations, rewards, dones, infos) with auto-reset."""
        masks = self._masks(actions)
        self._step_count += 1
        self._steps += 1
        self._launch(masks)
        ram_mode = self.observation_mode == "ram"
        copied = ram_mode or self.observation_cadence <= 1 or self._step_count % self.observation_cadence == 0
        # The info dicts do not depend on the step's results, so they are built
        # while the step runs on the GPU: one dict per env (SB3 adds keys per env).
        base = self._info(observation_cadence=self.observation_cadence, observations_copied=copied,
                          observations_stale=not copied,
                          rgb_observations_copied=copied and self.observation_mode == "rgb_array")
        infos = [base.copy() for _ in range(self.num_envs)]
        ram, rewards, dones = self._step_outputs(with_ram=ram_mode)
        if ram_mode:
            obs = ram
        elif copied:
            obs = self._frames()
            self._obs_cache = obs
        else:
            obs = self._obs_cache if self._obs_cache is not None else self._frames()
        dones, trunc = self._done_and_truncation(dones)
        if dones.any():
            idx = np.nonzero(dones)[0]
            for i in idx:
                infos[i]["terminal_observation"] = obs[i].copy()
                infos[i]["terminated"] = bool(not trunc[i])
                infos[i]["truncated"] = bool(trunc[i])
                self.reset_infos[i] = self._info()
            self._batch.reset_envs(dones.astype(np.uint8))
            obs = np.array(obs, copy=True) if not copied else obs
            obs[idx] = self._rows(idx)
            if self.observation_mode != "ram":
                self._obs_cache = obs
            self._steps[dones] = 0
        self._pending = None
        self.buf_infos = infos
        return obs, rewards, dones, infos

    def step_reward(self, actions: Iterable[int]):
        """Rewards and dones only (no observation copies); auto-reset as in step()."""
        masks = self._masks(actions)
        self._steps += 1
        self._launch(masks)
        base = self._info(observations_copied=False)
        infos = [base.copy() for _ in range(self.num_envs)]  # built while the step runs
        _, rewards, dones = self._step_outputs(with_ram=False)
        dones, trunc = self._done_and_truncation(dones)
        if dones.any():
            idx = np.nonzero(dones)[0]
            terminal = self._rows(idx)
            for k, i in enumerate(idx):
                infos[i]["terminal_observation"] = terminal[k].copy()
                infos[i]["terminated"] = bool(not trunc[i])
                infos[i]["truncated"] = bool(trunc[i])
                self.reset_infos[i] = self._info()
            self._batch.reset_envs(dones.astype(np.uint8))
            self._steps[dones] = 0
        self._pending = None
        self.buf_infos = infos
        return rewards, dones, infos

    def render(self, mode: str | None = "rgb_array") -> np.ndarray | None:
        if mode is None:
            return None
        if mode != "rgb_array":
            raise ValueError("only rgb_array rendering is supported")
        return np.asarray(self._batch.render(), np.uint8)

    def get_images(self) -> list[np.ndarray]:
        frames = self.render()
        return [frames[i].copy() for i in range(self.num_envs)]

    def close(self) -> None:
        self._batch = None
