"""GPU-resident PPO on the batched core (the consumer side of the env-step path).

Mirrors the reference's ``nesle.native_ppo`` (src/nesle/native_ppo.py): same
config names, the same rollout -> GAE -> clipped-surrogate update, with the
observation handed over by DLPack.  B200-first differences:

* no host synchronisation inside a rollout -- actions are sampled and mapped
  to joypad masks on the device, auto-reset is fused into the step kernel
  (the reference syncs every step to build a host reset mask,
  native_ppo.py:491-509), rewards and dones are read through device views;
* the policy is the benchmark's bf16 MLP (2048 RAM bytes / 255 -> 512 -> 256,
  ReLU, 7 logits + value), matmuls under bf16 autocast with fp32 master
  weights and Adam state;
* across GPUs (one process per GPU) the gradients are averaged with a single
  flattened NCCL all-reduce per minibatch.
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass
from typing import Any

import numpy as np

from . import workloads as w


@dataclass
class NativePPOConfig:
    num_envs: int = 2048
    n_steps: int = 128
    batch_size: int = 8192
    update_epochs: int = 4
    frameskip: int = 4
    learning_rate: float = 2.5e-4
    gamma: float = 0.99
    gae_lambda: float = 0.95
    clip_coef: float = 0.1
    ent_coef: float = 0.01
    vf_coef: float = 0.5
    max_grad_norm: float = 0.5
    hidden_sizes: tuple[int, int] = (512, 256)
    seed: int = 1


def make_model(obs_dim: int, action_dim: int, hidden_sizes: tuple[int, int], device):
    """RAM actor-critic: uint8 RAM / 255 -> Linear+ReLU -> Linear+ReLU -> (logits, value).
    Orthogonal init as in native_ppo.py:69-102."""
    import torch
    import torch.nn as nn

    h1, h2 = hidden_sizes

    class RamActorCritic(nn.Module):
        def __init__(self) -> None:
            super().__init__()
            self.net = nn.Sequential(nn.Linear(obs_dim, h1), nn.ReLU(), nn.Linear(h1, h2), nn.ReLU())
            self.actor = nn.Linear(h2, action_dim)
            self.critic = nn.Linear(h2, 1)
            for layer in self.net:
                if isinstance(layer, nn.Linear):
                    nn.init.orthogonal_(layer.weight, math.sqrt(2.0))
                    nn.init.zeros_(layer.bias)
            nn.init.orthogonal_(self.actor.weight, 0.01)
            nn.init.zeros_(self.actor.bias)
            nn.init.orthogonal_(self.critic.weight, 1.0)
            nn.init.zeros_(self.critic.bias)

        def forward(self, obs):
            with torch.autocast("cuda", dtype=torch.bfloat16, enabled=obs.is_cuda, cache_enabled=False):
                x = obs.to(torch.bfloat16 if obs.is_cuda else torch.float32) * (1.0 / 255.0)
                f = self.net(x)
                logits, value = self.actor(f), self.critic(f).squeeze(-1)
            return logits.float(), value.float()

    return RamActorCritic().to(device)


def compute_gae(rewards, dones, values, next_done, next_value, gamma: float, gae_lambda: float):
    """Generalised advantage estimation over a (T, N) rollout (native_ppo.py:626-640).
    ``dones[t]`` is the done flag observed before step t; returns (advantages, returns)."""
    import torch

    advantages = torch.zeros_like(rewards)
    lastgaelam = torch.zeros(rewards.shape[1], dtype=rewards.dtype, device=rewards.device)
    for t in reversed(range(rewards.shape[0])):
        if t == rewards.shape[0] - 1:
            next_nonterminal = 1.0 - next_done
            next_values = next_value
        else:
            next_nonterminal = 1.0 - dones[t + 1]
            next_values = values[t + 1]
        delta = rewards[t] + gamma * next_values * next_nonterminal - values[t]
        lastgaelam = delta + gamma * gae_lambda * next_nonterminal * lastgaelam
        advantages[t] = lastgaelam
    return advantages, advantages + values


def allreduce_mean_grads(params, world: int) -> None:
    """Average the gradients of `params` over the process group with one
    flattened all-reduce (NCCL on GPUs, gloo on CPU)."""
    import torch
    import torch.distributed as dist

    if world <= 1:
        return
    grads = [p.grad for p in params if p.grad is not None]
    flat = torch.cat([g.reshape(-1) for g in grads])
    dist.all_reduce(flat)
    flat.mul_(1.0 / world)
    off = 0
    for g in grads:
        n = g.numel()
        g.copy_(flat[off:off + n].view_as(g))
        off += n


def batch_snapshot_args(wl: w.Workload, env: np.ndarray) -> tuple:
    """(snapshot, env_to_level) for CudaBatch as env.py:349-358 passes them: none,
    one snapshot as bytes, or a list with the per-env level of the global env index."""
    if not wl.snapshots:
        return None, None
    if len(wl.snapshots) == 1:
        return wl.snapshots[0], None
    return wl.snapshots, wl.env_to_level(env)


class PPOTrainer:
    """One process (one GPU) of the GPU-resident PPO loop on a CudaBatch."""

    def __init__(self, config: NativePPOConfig, workload: w.Workload | None = None, *, device: int = 0,
                 rank: int = 0, world: int = 1, use_graphs: bool = True):
        import torch

        from ._cuda_core import CudaBatch

        self.cfg = config
        self.world = world
        self.rank = rank
        self.dev = torch.device("cuda", device)
        rollout = config.num_envs * config.n_steps
        if rollout < config.batch_size:
            raise ValueError(f"rollout produces {rollout} samples per update but batch_size={config.batch_size} "
                             "is larger")
        torch.manual_seed(config.seed + rank)
        wl = workload or w.config2(seed=config.seed)
        self.wl = wl
        offset = rank * config.num_envs
        env = np.arange(offset, offset + config.num_envs)
        self.batch = CudaBatch(config.num_envs, config.frameskip, wl.rom.image, *batch_snapshot_args(wl, env),
                               device=device, done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed,
                               env_offset=offset)
        self.batch.reset_device()
        self.mask_table = torch.tensor(w.SIMPLE_MOVEMENT_MASKS, dtype=torch.uint8, device=self.dev)
        self.model = make_model(2048, len(w.SIMPLE_MOVEMENT_MASKS), config.hidden_sizes, self.dev)
        if world > 1:  # identical initial weights on every rank
            import torch.distributed as dist

            for p in self.model.parameters():
                dist.broadcast(p.data, src=0)
        # CUDA-graph the minibatch update (capturable Adam keeps its step
        # counters on the device).  Across GPUs it is two graphs around one
        # NCCL all-reduce of a flat gradient buffer, so no collective is
        # captured.
        self.use_graphs = use_graphs
        self._split_graphs = world > 1
        self._graph = None
        self._eager_steps = 0
        self.opt = torch.optim.Adam(self.model.parameters(), lr=config.learning_rate, eps=1e-5,
                                    capturable=self.use_graphs)
        T, N = config.n_steps, config.num_envs
        self.obs_buf = torch.empty((T, N, 2048), dtype=torch.uint8, device=self.dev)
        self.act_buf = torch.empty((T, N), dtype=torch.long, device=self.dev)
        self.logp_buf = torch.empty((T, N), dtype=torch.float32, device=self.dev)
        self.rew_buf = torch.empty((T, N), dtype=torch.float32, device=self.dev)
        self.done_buf = torch.empty((T, N), dtype=torch.float32, device=self.dev)
        self.val_buf = torch.empty((T, N), dtype=torch.float32, device=self.dev)
        self.next_done = torch.zeros(N, dtype=torch.float32, device=self.dev)
        self.obs = torch.utils.dlpack.from_dlpack(self.batch.ram_device())  # (N, 2048) uint8, zero-copy
        self.rewards = torch.utils.dlpack.from_dlpack(self.batch.rewards_device())
        self.dones = torch.utils.dlpack.from_dlpack(self.batch.last_done_device())
        self.global_step = 0

    def rollout(self) -> None:
        """n_steps env-steps of every env; no host synchronisation."""
        import torch

        for t in range(self.cfg.n_steps):
            self.obs_buf[t].copy_(self.obs)  # the RAM view is updated in place by the next step
            self.done_buf[t].copy_(self.next_done)
            with torch.no_grad():
                logits, value = self.model(self.obs)
                logp_all = torch.log_softmax(logits, dim=-1)
                # Gumbel-max: a sample of the categorical with no host round trip
                u = torch.rand_like(logp_all).clamp_(1e-20, 1.0)
                action = torch.argmax(logp_all - torch.log(-torch.log(u)), dim=-1)
                self.logp_buf[t].copy_(logp_all.gather(1, action[:, None]).squeeze(1))
            self.act_buf[t].copy_(action)
            self.val_buf[t].copy_(value)
            self.batch.step_device(self.mask_table[action], auto_reset=True, synchronize=False)
            self.rew_buf[t].copy_(self.rewards)
            self.next_done.copy_(self.dones)
        self.global_step += self.cfg.num_envs * self.cfg.n_steps * self.world

    def _minibatch_loss(self, obs, act, logp, adv, ret):
        """Clipped-surrogate PPO loss of one minibatch (native_ppo.py:545-563)."""
        import torch

        cfg = self.cfg
        logits, newvalue = self.model(obs)
        logp_all = torch.log_softmax(logits, dim=-1)
        newlogp = logp_all.gather(1, act[:, None]).squeeze(1)
        entropy = -(logp_all.exp() * logp_all).sum(-1).mean()
        ratio = (newlogp - logp).exp()
        mb_adv = (adv - adv.mean()) / (adv.std() + 1e-8)
        pg_loss = torch.max(-mb_adv * ratio,
                            -mb_adv * torch.clamp(ratio, 1.0 - cfg.clip_coef, 1.0 + cfg.clip_coef)).mean()
        v_loss = 0.5 * (newvalue - ret).pow(2).mean()
        return pg_loss - cfg.ent_coef * entropy + cfg.vf_coef * v_loss

    def _eager_step(self, obs, act, logp, adv, ret):
        import torch

        params = list(self.model.parameters())
        loss = self._minibatch_loss(obs, act, logp, adv, ret)
        self.opt.zero_grad(set_to_none=True)
        loss.backward()
        allreduce_mean_grads(params, self.world)
        torch.nn.utils.clip_grad_norm_(params, self.cfg.max_grad_norm)
        self.opt.step()
        return loss.detach()

    def _graph_step(self, b, idx):
        """One minibatch update as CUDA graph replays: the minibatch is gathered
        into static buffers, then forward, backward, clipping and the Adam step
        replay from one captured graph.  With split graphs the gradients land in
        one flat buffer, which is all-reduced between the backward graph and the
        clip + Adam graph."""
        import torch
        import torch.distributed as dist

        g = self._graph
        for name, src in zip(("obs", "act", "logp", "adv", "ret"), b):
            torch.index_select(src, 0, idx, out=g[name])
        g["graph"].replay()
        if "step_graph" in g:
            if self.world > 1:
                dist.all_reduce(g["flat"])
            g["step_graph"].replay()
        return g["loss"].detach().clone()

    def _capture(self, b, idx):
        import torch

        params = list(self.model.parameters())
        static = {name: torch.index_select(src, 0, idx)
                  for name, src in zip(("obs", "act", "logp", "adv", "ret"), b)}
        graph = torch.cuda.CUDAGraph()
        if self._split_graphs:
            # every gradient a view of one flat buffer (backward accumulates into
            # it in place), so the all-reduce is one call on contiguous memory
            flat = torch.zeros(sum(p.numel() for p in params), dtype=params[0].dtype, device=self.dev)
            off = 0
            for p in params:
                p.grad = flat[off:off + p.numel()].view_as(p)
                off += p.numel()
            with torch.cuda.graph(graph):
                flat.zero_()
                loss = self._minibatch_loss(static["obs"], static["act"], static["logp"], static["adv"],
                                            static["ret"])
                loss.backward()
            step_graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(step_graph):
                flat.mul_(1.0 / self.world)
                torch.nn.utils.clip_grad_norm_(params, self.cfg.max_grad_norm)
                self.opt.step()
            static["flat"] = flat
            static["step_graph"] = step_graph
        else:
            self.opt.zero_grad(set_to_none=True)
            with torch.cuda.graph(graph):
                loss = self._minibatch_loss(static["obs"], static["act"], static["logp"], static["adv"],
                                            static["ret"])
                loss.backward()
                torch.nn.utils.clip_grad_norm_(params, self.cfg.max_grad_norm)
                self.opt.step()
        static["loss"] = loss
        static["graph"] = graph
        self._graph = static

    def update(self) -> dict[str, Any]:
        """GAE + update_epochs passes of clipped-surrogate minibatch updates.
        The minibatch step replays captured CUDA graphs after a few eager
        warm-up steps (across GPUs, two graphs around the NCCL all-reduce)."""
        import torch

        cfg = self.cfg
        with torch.no_grad():
            _, next_value = self.model(self.obs)
            adv, ret = compute_gae(self.rew_buf, self.done_buf, self.val_buf, self.next_done, next_value,
                                   cfg.gamma, cfg.gae_lambda)
        b = (self.obs_buf.reshape(-1, 2048), self.act_buf.reshape(-1), self.logp_buf.reshape(-1),
             adv.reshape(-1), ret.reshape(-1))
        count = b[0].shape[0]
        losses = []
        for _ in range(cfg.update_epochs):
            perm = torch.randperm(count, device=self.dev)
            for start in range(0, count, cfg.batch_size):
                idx = perm[start:start + cfg.batch_size]
                full = idx.shape[0] == cfg.batch_size  # a trailing partial minibatch steps eagerly
                if full and self._graph is not None:
                    losses.append(self._graph_step(b, idx))
                    continue
                if full and self.use_graphs and self._eager_steps >= 3:
                    torch.cuda.synchronize(self.dev)
                    self._capture(b, idx)
                    losses.append(self._graph_step(b, idx))
                    continue
                losses.append(self._eager_step(*(x[idx] for x in b)))
                self._eager_steps += 1
        return {"loss": torch.stack(losses).mean(), "samples": count}

    def iteration(self) -> dict[str, Any]:
        self.rollout()
        return self.update()


def train_native_ppo(config: NativePPOConfig, iterations: int, workload: w.Workload | None = None,
                     device: int = 0) -> list[float]:
    """Single-GPU training loop; returns the mean loss of every iteration."""
    trainer = PPOTrainer(config, workload, device=device)
    out = []
    t0 = time.perf_counter()
    for it in range(iterations):
        stats = trainer.iteration()
        out.append(float(stats["loss"]))
        fps = trainer.global_step / max(1e-9, time.perf_counter() - t0)
        print(f"iteration={it + 1}/{iterations} step={trainer.global_step} loss={out[-1]:.4f} fps={fps:.0f}",
              flush=True)
    trainer.batch.synchronize()
    return out
