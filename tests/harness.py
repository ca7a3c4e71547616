"""Uniform wrappers for the parity tests.

``HostCore`` drives the product kernel core compiled for the CPU
(tests/native/core_host.cpp); ``GpuCore`` drives libnesle_b200.so through its
C ABI on a CUDA device.  Both expose the checker's interface (``step``,
``reset``, ``reset_envs``, ``poke_ram``, ``render``, ``get(field)`` with the
checker's field names) so one comparison routine serves every pair.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

from nesle_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
NATIVE = ROOT / "tests" / "native"
HOST_SO = NATIVE / "_build" / "libcore_host.so"

# checker field name -> product field name
PRODUCT_NAME = {"nt": "nametable", "pal": "palette", "snap_nt": "snap_nametable", "snap_pal": "snap_palette",
                "reward": "rewards", "last_reward": "last_rewards"}

# Fields compared after every step.
STATE_FIELDS = ("pc", "a", "x", "y", "sp", "p", "cycles", "ram", "prg_ram", "frame", "frame_dot", "ppu_status",
                "ppu_ctrl", "ppu_mask", "nmi_pending", "oam", "oam_addr", "v", "t", "w", "fine_x", "open_bus",
                "read_buffer", "scroll_x", "scroll_y", "nt", "pal", "ctrl_shift", "ctrl_count", "ctrl_strobe",
                "reward", "last_reward", "done", "last_done", "prev_x", "prev_time", "episode", "status",
                "stat_instructions", "stat_frames", "stat_budget_hits", "lat_sx", "lat_sy", "lat_ctrl",
                "snap_sx_start", "snap_sy_start", "snap_ctrl_start", "snap_sx_end", "snap_sy_end",
                "snap_ctrl_end", "snap_mask", "snap_oam", "snap_nt", "snap_pal")


def build_host_core() -> Path:
    srcs = [NATIVE / "core_host.cpp", ROOT / "nesle_b200" / "csrc" / "formats.cpp"]
    deps = srcs + list((ROOT / "nesle_b200" / "csrc").glob("*.cuh")) + list((ROOT / "nesle_b200" / "csrc").glob("*.h"))
    if HOST_SO.exists() and all(d.stat().st_mtime <= HOST_SO.stat().st_mtime for d in deps):
        return HOST_SO
    HOST_SO.parent.mkdir(parents=True, exist_ok=True)
    subprocess.run(["g++", "-std=c++20", "-O2", "-fPIC", "-shared", "-I", str(ROOT / "include"), "-o", str(HOST_SO),
                    *map(str, srcs)], check=True)
    return HOST_SO


class _Common:
    num_envs: int

    def get(self, field: str) -> np.ndarray:
        name = PRODUCT_NAME.get(field, field)
        dtype, shape = _lib.FIELDS[name]
        out = np.zeros((self.num_envs, *shape), dtype=dtype)
        self._copy(name, out)
        return out


class HostCore(_Common):
    _h_lib = None
    global_ram = False  # subclass HostCoreGlobal runs the in-place RAM variant
    v2 = True           # the v2 datapath (nes_v2.cuh); the V1 subclasses run the first one
    early = 0           # v2: execution-entry quarters prefetched one iteration ahead (0-2)

    @classmethod
    def lib(cls):
        if cls._h_lib is None:
            lib = ctypes.CDLL(str(build_host_core()))
            lib.host_create.argtypes = [ctypes.POINTER(_lib.CreateArgs), ctypes.POINTER(ctypes.c_void_p)]
            lib.host_last_error.restype = ctypes.c_char_p
            lib.host_destroy.argtypes = [ctypes.c_void_p]
            lib.host_reset.argtypes = [ctypes.c_void_p]
            lib.host_reset_envs.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
            lib.host_poke_ram.argtypes = [ctypes.c_void_p, ctypes.c_uint16, ctypes.c_uint8]
            lib.host_step.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
            lib.host_render.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
            lib.host_copy_field.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_uint64]
            lib.host_set_global_ram.argtypes = [ctypes.c_void_p, ctypes.c_int]
            lib.host_set_v2.argtypes = [ctypes.c_void_p, ctypes.c_int]
            lib.host_set_early.argtypes = [ctypes.c_void_p, ctypes.c_int]
            cls._h_lib = lib
        return cls._h_lib

    def __init__(self, num_envs, frameskip, rom, snapshots=(), env_to_level=None, done_mode=0, done_args=(0, 0),
                 seed=0, env_offset=0):
        self.num_envs = num_envs
        args, keep = _lib.make_create_args(num_envs, frameskip, rom, snapshots, env_to_level, done_mode, done_args,
                                           seed, env_offset)
        h = ctypes.c_void_p()
        if self.lib().host_create(ctypes.byref(args), ctypes.byref(h)):
            raise ValueError(self.lib().host_last_error().decode())
        self._h = h
        self.lib().host_set_global_ram(h, int(self.global_ram))
        self.lib().host_set_v2(h, int(self.v2))
        self.lib().host_set_early(h, int(self.early))

    def __del__(self):
        if getattr(self, "_h", None):
            self.lib().host_destroy(self._h)
            self._h = None

    def reset(self):
        self.lib().host_reset(self._h)

    def reset_envs(self, mask):
        m = np.ascontiguousarray(mask, dtype=np.uint8)
        self.lib().host_reset_envs(self._h, m.ctypes.data)

    def poke_ram(self, address, value):
        self.lib().host_poke_ram(self._h, address, value)

    def step(self, actions, device_api=True, auto_reset=True):
        a = np.ascontiguousarray(actions, dtype=np.uint8)
        self.lib().host_step(self._h, a.ctypes.data, int(device_api), int(auto_reset))

    def render(self) -> dict:
        n = self.num_envs
        out = {"index": np.zeros((n, 240, 256), np.uint8), "rgb": np.zeros((n, 240, 256, 3), np.uint8),
               "gray84": np.zeros((n, 84, 84), np.uint8)}
        for mode, key in ((0, "rgb"), (1, "index"), (2, "gray84")):
            self.lib().host_render(self._h, mode, out[key].ctypes.data)
        return out

    def _copy(self, name, out):
        rc = self.lib().host_copy_field(self._h, name.encode(), out.ctypes.data, out.nbytes)
        if rc:
            raise KeyError(self.lib().host_last_error().decode())


class HostCoreGlobal(HostCore):
    global_ram = True


class HostCoreHybrid(HostCore):
    global_ram = 2  # in place, zero page in a separate slot


class HostCoreHybridStack(HostCore):
    global_ram = 3  # in place, stack page in a separate slot


class HostCoreEarly1(HostCore):
    early = 1  # shared RAM, one entry quarter prefetched


class HostCoreHybridEarly1(HostCore):
    global_ram = 2
    early = 1  # the interleaved placement's datapath: zero page in a slot, one quarter prefetched


class HostCoreHybridEarly2(HostCore):
    global_ram = 2
    early = 2  # the deepest prefetch the datapath supports


class HostCoreV1(HostCore):
    v2 = False  # RAM in the interleaved slot, first datapath


class HostCoreHybridV1(HostCore):
    global_ram = 2
    v2 = False


class HostCoreGlobalAsync(HostCore):
    global_ram = 4  # in place, operands loaded ahead (with idle iterations)


class HostCoreHybridAsync(HostCore):
    global_ram = 5  # hybrid, operands outside the zero page loaded ahead


class GpuCore(_Common):
    """libnesle_b200.so through its C ABI (host arrays in, host copies out)."""

    def __init__(self, num_envs, frameskip, rom, snapshots=(), env_to_level=None, done_mode=0, done_args=(0, 0),
                 seed=0, env_offset=0, device=0):
        self.lib = _lib.load()
        self.num_envs = num_envs
        args, keep = _lib.make_create_args(num_envs, frameskip, rom, snapshots, env_to_level, done_mode, done_args,
                                           seed, env_offset, device)
        h = ctypes.c_void_p()
        _lib.check(self.lib.nesle_create(ctypes.byref(args), ctypes.byref(h)))
        self._h = h

    def __del__(self):
        if getattr(self, "_h", None):
            self.lib.nesle_destroy(self._h)
            self._h = None

    def reset(self):
        _lib.check(self.lib.nesle_reset(self._h, None))

    def reset_envs(self, mask):
        m = np.ascontiguousarray(mask, dtype=np.uint8)
        _lib.check(self.lib.nesle_reset_envs(self._h, m.ctypes.data, 0, None))

    def poke_ram(self, address, value):
        _lib.check(self.lib.nesle_poke_ram(self._h, address, value, None))

    def step(self, actions, device_api=True, auto_reset=True):
        a = np.ascontiguousarray(actions, dtype=np.uint8)
        _lib.check(self.lib.nesle_step(self._h, a.ctypes.data, _lib.ACTIONS_U8, 0, int(device_api),
                                       int(auto_reset), None))

    def render(self) -> dict:
        out = {}
        for mode, key, field in ((_lib.RENDER_RGB, "rgb", "frames_rgb"), (_lib.RENDER_INDEX, "index", "frames_index"),
                                 (_lib.RENDER_GRAY84, "gray84", "obs_gray84")):
            _lib.check(self.lib.nesle_render(self._h, mode, None))
            dtype, shape = _lib.FIELDS[field]
            host = np.zeros((self.num_envs, *shape), dtype)
            self._copy(field, host)
            out[key] = host
        return out

    def _copy(self, name, out):
        _lib.check(self.lib.nesle_copy_field(self._h, name.encode(), out.ctypes.data, out.nbytes))

    def gray84(self) -> np.ndarray:
        """The 84x84 observations of every env (nesle_render + copy)."""
        _lib.check(self.lib.nesle_render(self._h, _lib.RENDER_GRAY84, None))
        return self.get("obs_gray84")

    def window(self, envs) -> dict:
        """Every state field of the listed envs, under the checker's field names,
        through one nesle_save_states call (a few KB per env instead of whole-batch
        copies)."""
        idx = np.ascontiguousarray(envs, dtype=np.uint32)
        blobs = np.zeros((len(idx), _lib.STATE_BYTES), np.uint8)
        _lib.check(self.lib.nesle_save_states(self._h, idx.ctypes.data, len(idx), 0, blobs.ctypes.data, 0, None))
        rec = blobs[:, :128].copy().view(_lib.ENV_RECORD_DTYPE).reshape(len(idx))
        out = {name: rec[name].copy() for name in _lib.ENV_RECORD_DTYPE.names if name != "flags"}
        checker_name = {v: k for k, v in PRODUCT_NAME.items()}
        for part in ("ram", "prg_ram", "nametable", "palette", "oam", "snap_nametable", "snap_palette", "snap_oam"):
            off, size = _lib.STATE_PARTS[part]
            out[checker_name.get(part, part)] = blobs[:, off:off + size].copy()
        off, _ = _lib.STATE_PARTS["out"]
        f = blobs[:, off:off + 8].copy().view(np.float32)
        out["reward"], out["last_reward"] = f[:, 0].copy(), f[:, 1].copy()
        out["done"], out["last_done"] = blobs[:, off + 8].copy(), blobs[:, off + 9].copy()
        return out


def window_of(ref, fields=STATE_FIELDS) -> dict:
    """The same dict from any core with get(field) (the checker)."""
    return {f: ref.get(f) for f in fields}


def assert_same_window(want: dict, got: dict, fields=STATE_FIELDS, label: str = "") -> None:
    for f in fields:
        a, b = want[f], got[f]
        if not np.array_equal(a, b):
            bad = np.nonzero((a != b).reshape(a.shape[0], -1).any(1))[0]
            raise AssertionError(f"{label} field {f}: {len(bad)} envs differ, first {bad[:8].tolist()}; "
                                 f"ref {a[bad[0]].ravel()[:16]} other {b[bad[0]].ravel()[:16]}")


def assert_same(ref, other, fields=STATE_FIELDS, label: str = "") -> None:
    for f in fields:
        a, b = ref.get(f), other.get(f)
        if not np.array_equal(a, b):
            bad = np.nonzero((a != b).reshape(a.shape[0], -1).any(1))[0]
            raise AssertionError(f"{label} field {f}: {len(bad)} envs differ, first {bad[:8].tolist()}; "
                                 f"ref {a[bad[0]].ravel()[:16]} other {b[bad[0]].ravel()[:16]}")


def run_lockstep(make, n: int, steps: int, auto_reset: bool, others, fields=STATE_FIELDS, oracle_cls=None,
                 env_offset: int = 0, check_every: int = 1):
    """Step the checker and every constructor in `others` on the same inputs, comparing state."""
    from oracle import Oracle

    wl = make()
    env = np.arange(n) + env_offset
    e2l = wl.env_to_level(env) if wl.env_to_level else None
    kw = dict(env_to_level=e2l, done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed, env_offset=env_offset)
    ref = (oracle_cls or Oracle)(n, wl.frameskip, wl.rom.image, wl.snapshots, **kw)
    sims = [cls(n, wl.frameskip, wl.rom.image, wl.snapshots, **kw) for cls in others]
    for s in sims:
        assert_same(ref, s, fields, f"{wl.name} after create")
    dones = 0
    for step in range(steps):
        act = wl.actions(env, step)
        ref.step(act, auto_reset=auto_reset)
        for s in sims:
            s.step(act, auto_reset=auto_reset)
        if (step + 1) % check_every == 0 or step == steps - 1:
            for s in sims:
                assert_same(ref, s, fields, f"{wl.name} step {step}")
        dones += int(ref.get("last_done").sum())
    return ref, sims, dones
