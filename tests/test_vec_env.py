"""Host VecEnv path (nesle_b200.vec_env.NesleVecEnv): the SB3 contract of the
reference's NesleVecEnv CUDA branch (src/nesle/env.py:552-716) -- auto-reset
with terminal observations, truncation at max_episode_steps, step_reward --
checked against a restatement of that contract on the checker.  On CPU the
batch is a checker-backed stand-in (host logic only); on the GPU it is the
real CudaBatch with its page-locked copies.
"""
from __future__ import annotations

import numpy as np
import pytest

from nesle_b200 import workloads as w
from nesle_b200.vec_env import NesleVecEnv
from oracle import Oracle

N = 12


def _workload():
    wl = w.config4()
    wl.done_args = (6, 20)  # episodes of 2-5 env-steps
    return wl


def _oracle(wl, n=N):
    env = np.arange(n)
    return Oracle(n, wl.frameskip, wl.rom.image, wl.snapshots, env_to_level=wl.env_to_level(env),
                  done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed)


class CheckerBatch:
    """The slice of the CudaBatch interface NesleVecEnv uses, on the checker."""

    name = "cuda-console"

    def __init__(self, wl, n=N):
        self.o = _oracle(wl, n)

    def reset_device(self):
        self.o.reset()

    def step(self, masks, render_frame=True, copy_obs=True):
        self.o.step(np.asarray(masks, np.uint8), device_api=False, auto_reset=False)

    def ram(self):
        return self.o.get("ram")

    def get_field(self, name):
        return {"rewards": lambda: self.o.get("reward"), "done": lambda: self.o.get("done"),
                "obs_gray84": lambda: self.o.render()["gray84"]}[name]()

    def reset_envs(self, mask):
        self.o.reset_envs(np.asarray(mask, np.uint8))

    def render(self):
        return self.o.render()["rgb"]

    def obs_gray84_device(self, render=True):
        return None


def _expected_run(wl, actions, masks, max_steps, mode):
    """The SB3 contract restated on a second checker."""
    o = _oracle(wl)
    o.reset()
    steps = np.zeros(N, np.int64)
    obs_fn = (lambda: o.get("ram")) if mode == "ram" else (lambda: o.render()["gray84"])
    out = []
    for a in actions:
        o.step(masks[a], device_api=False, auto_reset=False)
        steps += 1
        obs = obs_fn().copy()
        rew = o.get("reward").copy()
        trunc = steps >= max_steps if max_steps else np.zeros(N, bool)
        done = o.get("done").astype(bool) | trunc
        term = {int(i): obs[i].copy() for i in np.nonzero(done)[0]}
        if done.any():
            o.reset_envs(done.astype(np.uint8))
            fresh = obs_fn()
            obs[done] = fresh[done]
            steps[done] = 0
        out.append((obs, rew, done, term, trunc))
    return out


def _check(env, wl, mode, max_steps, n_steps=10):
    rng = np.random.default_rng(3)
    actions = [rng.integers(0, len(w.SIMPLE_MOVEMENT_MASKS), N) for _ in range(n_steps)]
    masks = np.asarray(w.SIMPLE_MOVEMENT_MASKS, np.uint8)
    expected = _expected_run(wl, actions, masks, max_steps, mode)
    obs0 = env.reset()
    assert obs0.shape == ((N, 2048) if mode == "ram" else (N, 84, 84))
    total_done = 0
    for a, (eobs, erew, edone, eterm, etrunc) in zip(actions, expected):
        obs, rew, done, infos = env.step(a)
        np.testing.assert_array_equal(obs, eobs)
        np.testing.assert_array_equal(rew, erew)
        np.testing.assert_array_equal(done, edone)
        for i, info in enumerate(infos):
            assert info["backend"] == "cuda-console" and info["observation_mode"] == mode
            if done[i]:
                np.testing.assert_array_equal(info["terminal_observation"], eterm[i])
                assert info["truncated"] == bool(etrunc[i]) and info["terminated"] == (not etrunc[i])
            else:
                assert "terminal_observation" not in info
        total_done += int(done.sum())
    assert total_done > N  # several episodes ended (and some by truncation when enabled)


@pytest.mark.parametrize("max_steps", [0, 3])
@pytest.mark.parametrize("mode", ["ram", "gray84"])
def test_contract_on_checker_batch(mode, max_steps):
    wl = _workload()
    env = NesleVecEnv(None, N, observation_mode=mode, max_episode_steps=max_steps, batch=CheckerBatch(wl))
    _check(env, wl, mode, max_steps)


def test_step_reward_and_argument_checks():
    wl = _workload()
    env = NesleVecEnv(None, N, batch=CheckerBatch(wl))
    env.reset()
    rew, done, infos = env.step_reward(np.zeros(N, np.int64))
    assert rew.shape == (N,) and done.dtype == bool and len(infos) == N
    with pytest.raises(ValueError):
        env.step(np.full(N, 7))  # 7 actions: indices 0-6
    with pytest.raises(ValueError):
        env.step(np.zeros(N - 1, np.int64))
    with pytest.raises(RuntimeError):
        env.step_wait()
    env.step_async(np.ones(N, np.int64))
    env.step_wait()
    with pytest.raises(ValueError):
        NesleVecEnv(None, N, observation_mode="hsv", batch=CheckerBatch(wl))


@pytest.mark.gpu
@pytest.mark.parametrize("max_steps", [0, 3])
@pytest.mark.parametrize("mode", ["ram", "gray84"])
def test_contract_on_gpu(mode, max_steps):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nesle_b200 import build

    build.build()
    wl = _workload()
    env = NesleVecEnv(wl.rom.image, N, observation_mode=mode, max_episode_steps=max_steps,
                      snapshots=wl.snapshots, env_to_level=wl.env_to_level(np.arange(N)),
                      done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed)
    _check(env, wl, mode, max_steps)
