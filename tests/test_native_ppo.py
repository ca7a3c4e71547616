"""GPU-resident PPO (nesle_b200.native_ppo), modelled on the reference's
tests/test_native_ppo.py: GAE against a float64 restatement, the model's
shapes, the gradient all-reduce over two gloo ranks on CPU, and on the GPU a
short training run whose environment side is replayed on the checker.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")


def _gae_numpy(rewards, dones, values, next_done, next_value, gamma, lam):
    T, _ = rewards.shape
    adv = np.zeros_like(rewards)
    last = np.zeros(rewards.shape[1])
    for t in reversed(range(T)):
        nnt = 1.0 - (next_done if t == T - 1 else dones[t + 1])
        nv = next_value if t == T - 1 else values[t + 1]
        delta = rewards[t] + gamma * nv * nnt - values[t]
        last = delta + gamma * lam * nnt * last
        adv[t] = last
    return adv, adv + values


def test_compute_gae_matches_float64_restatement():
    from nesle_b200.native_ppo import compute_gae

    rng = np.random.default_rng(0)
    T, N = 16, 9
    r = rng.normal(size=(T, N))
    d = (rng.random((T, N)) < 0.2).astype(np.float64)
    v = rng.normal(size=(T, N))
    nd = (rng.random(N) < 0.3).astype(np.float64)
    nv = rng.normal(size=N)
    ref_adv, ref_ret = _gae_numpy(r, d, v, nd, nv, 0.99, 0.95)
    f = lambda a: torch.tensor(a, dtype=torch.float32)  # noqa: E731
    adv, ret = compute_gae(f(r), f(d), f(v), f(nd), f(nv), 0.99, 0.95)
    np.testing.assert_allclose(adv.numpy(), ref_adv, rtol=1e-5, atol=1e-5)  # float32 vs float64
    np.testing.assert_allclose(ret.numpy(), ref_ret, rtol=1e-5, atol=1e-5)


def test_model_shapes_and_scaling_on_cpu():
    from nesle_b200.native_ppo import make_model

    m = make_model(2048, 7, (512, 256), "cpu")
    obs = torch.randint(0, 256, (5, 2048), dtype=torch.uint8)
    logits, value = m(obs)
    assert logits.shape == (5, 7) and value.shape == (5,) and logits.dtype == torch.float32
    assert [p.shape for p in m.net.parameters()][0] == (512, 2048)
    assert torch.isfinite(logits).all() and torch.isfinite(value).all()


def _grad_worker(rank, world, port, out_dir):
    import torch.distributed as dist

    from nesle_b200.native_ppo import allreduce_mean_grads

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        p1 = torch.nn.Parameter(torch.zeros(3, 4))
        p2 = torch.nn.Parameter(torch.zeros(5))
        p1.grad = torch.full((3, 4), float(rank + 1))
        p2.grad = torch.arange(5, dtype=torch.float32) * (rank + 1)
        allreduce_mean_grads([p1, p2], world)
        mean = sum(range(1, world + 1)) / world
        assert torch.allclose(p1.grad, torch.full((3, 4), mean))
        assert torch.allclose(p2.grad, torch.arange(5, dtype=torch.float32) * mean)
        if rank == 0:
            open(os.path.join(out_dir, "ok"), "w").write("ok")
    finally:
        dist.destroy_process_group()


def test_gradient_allreduce_two_gloo_ranks(tmp_path):
    mp = pytest.importorskip("torch.multiprocessing")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_grad_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    assert (tmp_path / "ok").read_text() == "ok"


@pytest.mark.gpu
def test_training_runs_and_env_side_replays_on_checker():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nesle_b200 import build
    from nesle_b200 import workloads as w
    from nesle_b200.native_ppo import NativePPOConfig, PPOTrainer
    from oracle import Oracle

    build.build()
    cfg = NativePPOConfig(num_envs=64, n_steps=8, batch_size=256, update_epochs=2)
    tr = PPOTrainer(cfg)
    wl = tr.wl
    o = Oracle(cfg.num_envs, cfg.frameskip, wl.rom.image, wl.snapshots, done_mode=wl.done_mode,
               done_args=wl.done_args, seed=wl.seed)
    masks = np.asarray(w.SIMPLE_MOVEMENT_MASKS, np.uint8)
    for _ in range(2):
        tr.rollout()
        acts = tr.act_buf.cpu().numpy()
        obs = tr.obs_buf.cpu().numpy()
        rews = tr.rew_buf.cpu().numpy()
        for t in range(cfg.n_steps):
            np.testing.assert_array_equal(obs[t], o.get("ram"), err_msg=f"obs before step {t}")
            o.step(masks[acts[t]])
            np.testing.assert_array_equal(rews[t], o.get("last_reward"))
        stats = tr.update()
        assert np.isfinite(float(stats["loss"]))
    np.testing.assert_array_equal(tr.batch.ram(), o.get("ram"))
    assert len(np.unique(tr.act_buf.cpu().numpy())) > 1  # the policy samples several actions


@pytest.mark.gpu
@pytest.mark.parametrize("split", [False, True])
def test_graphed_update_matches_eager_update(split):
    """The CUDA-graph update replays the eager minibatch step: one graph (one
    GPU), or the two graphs that run around the gradient all-reduce across GPUs
    (split, here with a world of one)."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nesle_b200 import build
    from nesle_b200.native_ppo import NativePPOConfig, PPOTrainer

    build.build()
    cfg = NativePPOConfig(num_envs=64, n_steps=16, batch_size=128, update_epochs=2)
    out = []
    for graphs in (False, True):
        tr = PPOTrainer(cfg, use_graphs=graphs)  # reseeds: identical init and rollout
        tr._split_graphs = split
        tr.rollout()
        stats = tr.update()
        out.append((tr.obs_buf.cpu(), float(stats["loss"]), [p.detach().cpu() for p in tr.model.parameters()],
                    tr._graph is not None))
    (obs_e, loss_e, par_e, g_e), (obs_g, loss_g, par_g, g_g) = out
    assert not g_e and g_g  # the second trainer really replayed a graph
    assert torch.equal(obs_e, obs_g)
    # float tolerance: bf16 autocast, and Adam's capturable and eager formulas round differently
    assert abs(loss_e - loss_g) <= 1e-3 * max(1.0, abs(loss_e))
    for a, b in zip(par_e, par_g):
        torch.testing.assert_close(a, b, rtol=1e-3, atol=5e-4)
