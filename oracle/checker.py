"""ctypes front-end for the two CPU checkers (test infrastructure only)."""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path
from typing import Sequence

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "liboracle.so"
REF_SO = HERE / "_ref" / "libnesle_ref.so"

# field -> (dtype, per-env shape)
FIELD_DTYPES: dict[str, tuple[np.dtype, tuple[int, ...]]] = {
    "pc": (np.uint16, ()), "a": (np.uint8, ()), "x": (np.uint8, ()), "y": (np.uint8, ()),
    "sp": (np.uint8, ()), "p": (np.uint8, ()), "cycles": (np.uint64, ()),
    "ctrl_shift": (np.uint8, ()), "ctrl_count": (np.uint8, ()), "ctrl_strobe": (np.uint8, ()),
    "pending_dma": (np.uint32, ()), "ppu_ctrl": (np.uint8, ()), "ppu_mask": (np.uint8, ()),
    "ppu_status": (np.uint8, ()), "oam_addr": (np.uint8, ()), "nmi_pending": (np.uint8, ()),
    "frame_dot": (np.uint32, ()), "frame": (np.uint64, ()), "v": (np.uint16, ()), "t": (np.uint16, ()),
    "fine_x": (np.uint8, ()), "w": (np.uint8, ()), "open_bus": (np.uint8, ()),
    "read_buffer": (np.uint8, ()), "scroll_x": (np.uint8, ()), "scroll_y": (np.uint8, ()),
    "lat_sx": (np.uint8, ()), "lat_sy": (np.uint8, ()), "lat_ctrl": (np.uint8, ()),
    "snap_sx_start": (np.uint8, ()), "snap_sy_start": (np.uint8, ()), "snap_ctrl_start": (np.uint8, ()),
    "snap_sx_end": (np.uint8, ()), "snap_sy_end": (np.uint8, ()), "snap_ctrl_end": (np.uint8, ()),
    "snap_mask": (np.uint8, ()), "prev_x": (np.int32, ()), "prev_time": (np.int32, ()),
    "reward": (np.float32, ()), "last_reward": (np.float32, ()), "done": (np.uint8, ()),
    "last_done": (np.uint8, ()), "action": (np.uint8, ()), "episode": (np.uint32, ()),
    "status": (np.uint32, ()), "stat_instructions": (np.uint64, ()), "stat_frames": (np.uint32, ()),
    "stat_budget_hits": (np.uint32, ()), "ram": (np.uint8, (2048,)), "prg_ram": (np.uint8, (8192,)),
    "nt": (np.uint8, (2048,)), "pal": (np.uint8, (32,)), "oam": (np.uint8, (256,)),
    "snap_oam": (np.uint8, (256,)), "snap_nt": (np.uint8, (2048,)), "snap_pal": (np.uint8, (32,)),
    "ram_touch": (np.uint64, ()), "prg_bank": (np.uint8, ()), "chr_bank": (np.uint8, ()),
    "snap_chr_bank": (np.uint8, ()),
}

_u8p = ctypes.POINTER(ctypes.c_uint8)


def build(quiet: bool = True) -> None:
    """Compile the checker (and the reference harness when the reference tree exists)."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True,
                   stdout=subprocess.DEVNULL if quiet else None)


def reference_available() -> bool:
    return REF_SO.exists()


def _bytes_array(items: Sequence[bytes]):
    bufs = [ctypes.create_string_buffer(b, len(b)) for b in items]
    ptrs = (ctypes.POINTER(ctypes.c_uint8) * max(1, len(items)))()
    for i, b in enumerate(bufs):
        ptrs[i] = ctypes.cast(b, _u8p)
    lens = (ctypes.c_size_t * max(1, len(items)))(*[len(b) for b in items])
    return bufs, ptrs, lens


def _as_u8(a: np.ndarray):
    return a.ctypes.data_as(_u8p)


class _Base:
    num_envs: int

    def get(self, field: str) -> np.ndarray:
        dtype, shape = FIELD_DTYPES[field]
        out = np.zeros((self.num_envs, *shape), dtype=dtype)
        self._get(field, out)
        return out

    def state_digest_fields(self) -> tuple[str, ...]:
        return ("pc", "a", "x", "y", "sp", "p", "cycles", "ram", "frame", "frame_dot",
                "ppu_status", "reward", "done")


class Oracle(_Base):
    """The C restatement (nes_oracle.c)."""

    _lib = None

    @classmethod
    def lib(cls):
        if cls._lib is None:
            if not ORACLE_SO.exists():
                build()
            lib = ctypes.CDLL(str(ORACLE_SO))
            lib.oracle_create.restype = ctypes.c_void_p
            lib.oracle_create.argtypes = [ctypes.c_uint32, ctypes.c_uint32, _u8p, ctypes.c_size_t,
                                          ctypes.POINTER(_u8p), ctypes.POINTER(ctypes.c_size_t),
                                          ctypes.c_uint32, _u8p, ctypes.c_uint32, ctypes.c_uint32,
                                          ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint32]
            lib.oracle_last_error.restype = ctypes.c_char_p
            for name in ("oracle_destroy", "oracle_reset"):
                getattr(lib, name).argtypes = [ctypes.c_void_p]
            lib.oracle_reset_envs.argtypes = [ctypes.c_void_p, _u8p]
            lib.oracle_step.argtypes = [ctypes.c_void_p, _u8p, ctypes.c_int, ctypes.c_int]
            lib.oracle_poke_ram.argtypes = [ctypes.c_void_p, ctypes.c_uint16, ctypes.c_uint8]
            lib.oracle_render.argtypes = [ctypes.c_void_p, _u8p, _u8p, _u8p]
            lib.oracle_get_field.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p]
            lib.oracle_get_field.restype = ctypes.c_int
            lib.oracle_decode_table.argtypes = [_u8p, _u8p, _u8p]
            lib.oracle_set_trace.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p,
                                             ctypes.c_uint32]
            lib.oracle_trace_count.restype = ctypes.c_uint32
            lib.oracle_trace_count.argtypes = [ctypes.c_void_p]
            lib.oracle_set_profile.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
            lib.oracle_counter_rand.restype = ctypes.c_uint64
            lib.oracle_counter_rand.argtypes = [ctypes.c_uint64, ctypes.c_uint32, ctypes.c_uint64,
                                                ctypes.c_uint64]
            cls._lib = lib
        return cls._lib

    def __init__(self, num_envs: int, frameskip: int, rom: bytes, snapshots: Sequence[bytes] = (),
                 env_to_level: np.ndarray | None = None, done_mode: int = 0,
                 done_args: tuple[int, int] = (0, 0), seed: int = 0, env_offset: int = 0):
        lib = self.lib()
        self.num_envs = num_envs
        rom_buf = ctypes.create_string_buffer(rom, len(rom))
        _keep, ptrs, lens = _bytes_array(list(snapshots))
        e2l = None if env_to_level is None else np.ascontiguousarray(env_to_level, dtype=np.uint8)
        self._h = lib.oracle_create(num_envs, frameskip, ctypes.cast(rom_buf, _u8p), len(rom), ptrs, lens,
                                    len(snapshots), None if e2l is None else _as_u8(e2l), done_mode,
                                    done_args[0], done_args[1], seed, env_offset)
        if not self._h:
            raise ValueError(lib.oracle_last_error().decode())

    def __del__(self):
        if getattr(self, "_h", None):
            self.lib().oracle_destroy(self._h)
            self._h = None

    def reset(self) -> None:
        self.lib().oracle_reset(self._h)

    def reset_envs(self, mask: np.ndarray) -> None:
        m = np.ascontiguousarray(mask, dtype=np.uint8)
        self.lib().oracle_reset_envs(self._h, _as_u8(m))

    def step(self, actions: np.ndarray, device_api: bool = True, auto_reset: bool = True) -> None:
        a = np.ascontiguousarray(actions, dtype=np.uint8)
        assert a.shape == (self.num_envs,)
        self.lib().oracle_step(self._h, _as_u8(a), int(device_api), int(auto_reset))

    def poke_ram(self, address: int, value: int) -> None:
        self.lib().oracle_poke_ram(self._h, address, value)

    def step_profile(self, actions: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
        """Host step (no auto-reset) returning the (256,) opcode and (65536,)
        fetch-address histograms of its instructions."""
        ops, pcs = np.zeros(256, np.uint64), np.zeros(65536, np.uint64)
        self.lib().oracle_set_profile(self._h, ops.ctypes.data, pcs.ctypes.data)
        try:
            self.step(actions, device_api=False, auto_reset=False)
        finally:
            self.lib().oracle_set_profile(self._h, None, None)
        return ops, pcs

    TRACE_DTYPE = np.dtype([("pc", "<u2"), ("op", "u1"), ("a", "u1"), ("x", "u1"), ("y", "u1"),
                            ("p", "u1"), ("sp", "u1"), ("cycles", "<u8")])

    def step_traced(self, actions: np.ndarray, env: int, cap: int = 400000,
                    device_api: bool = True, auto_reset: bool = True) -> np.ndarray:
        """step() while recording every instruction env `env` executes."""
        lib = self.lib()
        buf = np.zeros(cap, dtype=self.TRACE_DTYPE)
        lib.oracle_set_trace(self._h, env, buf.ctypes.data, cap)
        self.step(actions, device_api, auto_reset)
        n = lib.oracle_trace_count(self._h)
        lib.oracle_set_trace(self._h, 0, None, 0)
        return buf[:n]

    def render(self) -> dict[str, np.ndarray]:
        n = self.num_envs
        idx = np.zeros((n, 240, 256), np.uint8)
        rgb = np.zeros((n, 240, 256, 3), np.uint8)
        gray = np.zeros((n, 84, 84), np.uint8)
        self.lib().oracle_render(self._h, _as_u8(idx), _as_u8(rgb), _as_u8(gray))
        return {"index": idx, "rgb": rgb, "gray84": gray}

    def _get(self, field: str, out: np.ndarray) -> None:
        rc = self.lib().oracle_get_field(self._h, field.encode(), out.ctypes.data)
        if rc:
            raise KeyError(field)

    @classmethod
    def decode_table(cls) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        m, c, f = (np.zeros(256, np.uint8) for _ in range(3))
        cls.lib().oracle_decode_table(_as_u8(m), _as_u8(c), _as_u8(f))
        return m, c, f

    @classmethod
    def counter_rand(cls, seed: int, stream: int, a: int, b: int) -> int:
        return int(cls.lib().oracle_counter_rand(seed, stream, a, b))


class RefFcs(ctypes.Structure):
    _fields_ = [("pc", ctypes.c_uint16), ("v", ctypes.c_uint16), ("t", ctypes.c_uint16),
                ("a", ctypes.c_uint8), ("x", ctypes.c_uint8), ("y", ctypes.c_uint8), ("sp", ctypes.c_uint8),
                ("p", ctypes.c_uint8), ("ctrl", ctypes.c_uint8), ("mask", ctypes.c_uint8),
                ("status", ctypes.c_uint8), ("oam_addr", ctypes.c_uint8), ("open_bus", ctypes.c_uint8),
                ("read_buffer", ctypes.c_uint8), ("fine_x", ctypes.c_uint8), ("w", ctypes.c_uint8),
                ("ram", ctypes.c_uint8 * 2048), ("prg_ram", ctypes.c_uint8 * 8192),
                ("nt", ctypes.c_uint8 * 2048), ("pal", ctypes.c_uint8 * 32), ("oam", ctypes.c_uint8 * 256)]


class Reference(_Base):
    """The reference's own sources, compiled unchanged into oracle/_ref/."""

    _lib = None

    @classmethod
    def lib(cls):
        if cls._lib is None:
            if not REF_SO.exists():
                raise FileNotFoundError(f"{REF_SO} not built (needs the reference tree)")
            lib = ctypes.CDLL(str(REF_SO))
            lib.ref_create.restype = ctypes.c_void_p
            lib.ref_create.argtypes = [ctypes.c_char, ctypes.c_uint32, ctypes.c_uint32, _u8p, ctypes.c_size_t,
                                       ctypes.POINTER(_u8p), ctypes.POINTER(ctypes.c_size_t), ctypes.c_uint32,
                                       _u8p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                       ctypes.c_uint64, ctypes.c_uint32]
            lib.ref_last_error.restype = ctypes.c_char_p
            lib.ref_destroy.argtypes = [ctypes.c_void_p]
            lib.ref_reset.argtypes = [ctypes.c_void_p]
            lib.ref_reset_envs.argtypes = [ctypes.c_void_p, _u8p]
            lib.ref_step.argtypes = [ctypes.c_void_p, _u8p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
            lib.ref_render_rgb.argtypes = [ctypes.c_void_p, _u8p]
            lib.ref_get_field.argtypes = [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p]
            lib.ref_decode_table.argtypes = [_u8p, _u8p, _u8p]
            lib.ref_parse_fcs.argtypes = [_u8p, ctypes.c_size_t, ctypes.POINTER(RefFcs)]
            lib.ref_set_profile.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
            lib.ref_set_profile.restype = ctypes.c_int
            for f in ("ref_reset", "ref_reset_envs", "ref_step", "ref_render_rgb", "ref_get_field",
                      "ref_parse_fcs"):
                getattr(lib, f).restype = ctypes.c_int
            cls._lib = lib
        return cls._lib

    def __init__(self, kind: str, num_envs: int, frameskip: int, rom: bytes,
                 snapshots: Sequence[bytes] = (), env_to_level: np.ndarray | None = None,
                 done_mode: int = 0, done_args: tuple[int, int] = (0, 0), seed: int = 0,
                 env_offset: int = 0, threads: int = 1):
        lib = self.lib()
        self.kind = kind
        self.num_envs = num_envs
        self.threads = threads
        rom_buf = ctypes.create_string_buffer(rom, len(rom))
        _keep, ptrs, lens = _bytes_array(list(snapshots))
        e2l = None if env_to_level is None else np.ascontiguousarray(env_to_level, dtype=np.uint8)
        self._h = lib.ref_create(kind.encode(), num_envs, frameskip, ctypes.cast(rom_buf, _u8p), len(rom),
                                 ptrs, lens, len(snapshots), None if e2l is None else _as_u8(e2l),
                                 done_mode, done_args[0], done_args[1], seed, env_offset)
        if not self._h:
            raise ValueError(lib.ref_last_error().decode())

    def __del__(self):
        if getattr(self, "_h", None):
            self.lib().ref_destroy(self._h)
            self._h = None

    def _check(self, rc: int) -> None:
        if rc:
            raise RuntimeError(self.lib().ref_last_error().decode())

    def reset(self) -> None:
        self._check(self.lib().ref_reset(self._h))

    def reset_envs(self, mask: np.ndarray) -> None:
        m = np.ascontiguousarray(mask, dtype=np.uint8)
        self._check(self.lib().ref_reset_envs(self._h, _as_u8(m)))

    def step(self, actions: np.ndarray, device_api: bool = True, auto_reset: bool = True) -> None:
        a = np.ascontiguousarray(actions, dtype=np.uint8)
        assert a.shape == (self.num_envs,)
        self._check(self.lib().ref_step(self._h, _as_u8(a), int(device_api), int(auto_reset), self.threads))

    def step_profile(self, actions: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
        """Kind B: host step with the reference kernel's opcode / PC histograms."""
        ops, pcs = np.zeros(256, np.uint64), np.zeros(65536, np.uint64)
        self._check(self.lib().ref_set_profile(self._h, ops.ctypes.data, pcs.ctypes.data))
        try:
            self.step(actions, device_api=False, auto_reset=False)
        finally:
            self._check(self.lib().ref_set_profile(self._h, None, None))
        return ops, pcs

    def render_rgb(self) -> np.ndarray:
        out = np.zeros((self.num_envs, 240, 256, 3), np.uint8)
        self._check(self.lib().ref_render_rgb(self._h, _as_u8(out)))
        return out

    def _get(self, field: str, out: np.ndarray) -> None:
        self._check(self.lib().ref_get_field(self._h, field.encode(), out.ctypes.data))

    @classmethod
    def decode_table(cls) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        m, c, f = (np.zeros(256, np.uint8) for _ in range(3))
        cls.lib().ref_decode_table(_as_u8(m), _as_u8(c), _as_u8(f))
        return m, c, f

    @classmethod
    def parse_fcs(cls, data: bytes) -> dict:
        out = RefFcs()
        buf = ctypes.create_string_buffer(data, len(data))
        rc = cls.lib().ref_parse_fcs(ctypes.cast(buf, _u8p), len(data), ctypes.byref(out))
        if rc:
            raise RuntimeError(cls.lib().ref_last_error().decode())
        d = {name: getattr(out, name) for name, _ in RefFcs._fields_}
        for k in ("ram", "prg_ram", "nt", "pal", "oam"):
            d[k] = bytes(d[k])
        return d


def default_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))
