"""ctypes binding of libnesle_b200.so (include/nesle_b200.h).

Loading fails loudly: there is no CPU fallback.  The library is built in-tree
by ``python -m nesle_b200.build`` (``__graft_entry__.build()``).
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

PKG = Path(__file__).resolve().parent
LIB_PATH = PKG / "libnesle_b200.so"

NESLE_OK, NESLE_ERR_INVALID, NESLE_ERR_RUNTIME, NESLE_ERR_CUDA = 0, 1, 2, 3
DONE_SMB, DONE_RAM_EQ, DONE_FRAME_LIMIT = 0, 1, 2
ACTIONS_U8, ACTIONS_I64 = 0, 1
RENDER_RGB, RENDER_INDEX, RENDER_GRAY84 = 0, 1, 2
PTR_RAM, PTR_LAST_REWARDS, PTR_LAST_DONE, PTR_FRAMES_RGB, PTR_FRAMES_INDEX, PTR_OBS_GRAY84, PTR_REWARDS, \
    PTR_DONE = range(8)

_u8p = ctypes.POINTER(ctypes.c_uint8)


class CreateArgs(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("num_envs", ctypes.c_uint32), ("frameskip", ctypes.c_uint32),
                ("rom", _u8p), ("rom_len", ctypes.c_size_t), ("snapshots", ctypes.POINTER(_u8p)),
                ("snapshot_lens", ctypes.POINTER(ctypes.c_size_t)), ("num_snapshots", ctypes.c_uint32),
                ("env_to_level", _u8p), ("done_mode", ctypes.c_uint32), ("done_a", ctypes.c_uint32),
                ("done_b", ctypes.c_uint32), ("seed", ctypes.c_uint64), ("env_offset", ctypes.c_uint32),
                ("max_instructions_per_frame", ctypes.c_uint32)]


class Info(ctypes.Structure):
    _fields_ = [("num_envs", ctypes.c_uint32), ("frameskip", ctypes.c_uint32), ("num_levels", ctypes.c_uint32),
                ("device", ctypes.c_uint32), ("envs_per_block", ctypes.c_uint32),
                ("smem_bytes_per_block", ctypes.c_uint32), ("step_placement", ctypes.c_uint32)]


PLACEMENTS = ("shared", "global", "hybrid", "hybrid-stack", "global-async", "hybrid-async", "interleaved",
              "interleaved-async", "global-preload", "hybrid-preload", "interleaved-preload")


class FcsState(ctypes.Structure):
    _fields_ = [("pc", ctypes.c_uint16), ("a", ctypes.c_uint8), ("x", ctypes.c_uint8), ("y", ctypes.c_uint8),
                ("sp", ctypes.c_uint8), ("p", ctypes.c_uint8), ("cycles", ctypes.c_uint64),
                ("ppu_ctrl", ctypes.c_uint8), ("ppu_mask", ctypes.c_uint8), ("ppu_status", ctypes.c_uint8),
                ("ppu_oam_addr", ctypes.c_uint8), ("ppu_open_bus", ctypes.c_uint8),
                ("ppu_read_buffer", ctypes.c_uint8), ("ppu_x", ctypes.c_uint8), ("ppu_w", ctypes.c_uint8),
                ("ppu_v", ctypes.c_uint16), ("ppu_t", ctypes.c_uint16),
                ("cpu_ram", ctypes.c_uint8 * 2048), ("prg_ram", ctypes.c_uint8 * 8192),
                ("nametable_ram", ctypes.c_uint8 * 2048), ("palette_ram", ctypes.c_uint8 * 32),
                ("oam", ctypes.c_uint8 * 256)]


# Exported symbols and their ctypes signatures (every function include/nesle_b200.h declares).
SIGNATURES = {
    "nesle_create": (ctypes.c_int, [ctypes.POINTER(CreateArgs), ctypes.POINTER(ctypes.c_void_p)]),
    "nesle_destroy": (ctypes.c_int, [ctypes.c_void_p]),
    "nesle_reset": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "nesle_reset_envs": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "nesle_step": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                  ctypes.c_int, ctypes.c_void_p]),
    "nesle_step_profile": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                          ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    "nesle_host_alloc": (ctypes.c_int, [ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p)]),
    "nesle_host_free": (ctypes.c_int, [ctypes.c_void_p]),
    "nesle_state_bytes": (ctypes.c_uint64, []),
    "nesle_save_states": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int,
                                         ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "nesle_load_states": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int,
                                         ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "nesle_render": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "nesle_render_copy": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_uint64,
                                         ctypes.c_void_p]),
    "nesle_render_gray84_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint64,
                                                   ctypes.c_void_p]),
    "nesle_poke_ram": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint16, ctypes.c_uint8, ctypes.c_void_p]),
    "nesle_device_ptr": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p),
                                        ctypes.POINTER(ctypes.c_uint64)]),
    "nesle_copy_field": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_uint64]),
    "nesle_sync": (ctypes.c_int, [ctypes.c_void_p]),
    "nesle_stream_wait": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p]),
    "nesle_fault_count": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]),
    "nesle_get_info": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(Info)]),
    "nesle_parse_fcs": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(FcsState)]),
    "nesle_last_error": (ctypes.c_char_p, []),
    "nesle_abi_version": (ctypes.c_int, []),
}

# EnvRecord (csrc/nesle_state.h), the first 128 bytes of a saved state blob.
_REC = [("pc", "<u2", 0), ("a", "u1", 2), ("x", "u1", 3), ("y", "u1", 4), ("sp", "u1", 5), ("p", "u1", 6),
        ("nmi_pending", "u1", 7), ("cycles", "<u8", 8), ("frame", "<u8", 16), ("frame_dot", "<u4", 24),
        ("ppu_ctrl", "u1", 28), ("ppu_mask", "u1", 29), ("ppu_status", "u1", 30), ("oam_addr", "u1", 31),
        ("v", "<u2", 32), ("t", "<u2", 34), ("fine_x", "u1", 36), ("w", "u1", 37), ("open_bus", "u1", 38),
        ("read_buffer", "u1", 39), ("scroll_x", "u1", 40), ("scroll_y", "u1", 41), ("lat_sx", "u1", 42),
        ("lat_sy", "u1", 43), ("lat_ctrl", "u1", 44), ("snap_sx_start", "u1", 45), ("snap_sy_start", "u1", 46),
        ("snap_ctrl_start", "u1", 47), ("snap_sx_end", "u1", 48), ("snap_sy_end", "u1", 49),
        ("snap_ctrl_end", "u1", 50), ("snap_mask", "u1", 51), ("ctrl_shift", "u1", 52), ("ctrl_count", "u1", 53),
        ("ctrl_strobe", "u1", 54), ("flags", "u1", 55), ("prev_x", "<i4", 56), ("prev_time", "<i4", 60),
        ("pending_dma", "<u4", 64), ("episode", "<u4", 68), ("status", "<u4", 72),
        ("stat_instructions", "<u8", 80), ("stat_frames", "<u4", 88), ("stat_budget_hits", "<u4", 92)]
ENV_RECORD_DTYPE = np.dtype({"names": [n for n, _, _ in _REC], "formats": [f for _, f, _ in _REC],
                             "offsets": [o for _, _, o in _REC], "itemsize": 128})

# Saved-state blob parts: name -> (offset, bytes); see nesle_save_states.
STATE_PARTS = {"rec": (0, 128), "ram": (128, 2048), "prg_ram": (2176, 8192), "nametable": (10368, 2048),
               "palette": (12416, 32), "oam": (12448, 256), "snap_nametable": (12704, 2048),
               "snap_palette": (14752, 32), "snap_oam": (14784, 256), "out": (15040, 16)}
STATE_BYTES = 15056

# Per-env fields of nesle_copy_field: name -> (dtype, per-env shape).
FIELDS: dict[str, tuple[type, tuple[int, ...]]] = {
    "ram": (np.uint8, (2048,)), "prg_ram": (np.uint8, (8192,)), "nametable": (np.uint8, (2048,)),
    "palette": (np.uint8, (32,)), "oam": (np.uint8, (256,)), "snap_nametable": (np.uint8, (2048,)),
    "snap_palette": (np.uint8, (32,)), "snap_oam": (np.uint8, (256,)), "rewards": (np.float32, ()),
    "done": (np.uint8, ()), "last_rewards": (np.float32, ()), "last_done": (np.uint8, ()),
    "pc": (np.uint16, ()), "a": (np.uint8, ()), "x": (np.uint8, ()), "y": (np.uint8, ()), "sp": (np.uint8, ()),
    "p": (np.uint8, ()), "nmi_pending": (np.uint8, ()), "cycles": (np.uint64, ()), "frame": (np.uint64, ()),
    "frame_dot": (np.uint32, ()), "ppu_ctrl": (np.uint8, ()), "ppu_mask": (np.uint8, ()),
    "ppu_status": (np.uint8, ()), "oam_addr": (np.uint8, ()), "v": (np.uint16, ()), "t": (np.uint16, ()),
    "fine_x": (np.uint8, ()), "w": (np.uint8, ()), "open_bus": (np.uint8, ()), "read_buffer": (np.uint8, ()),
    "scroll_x": (np.uint8, ()), "scroll_y": (np.uint8, ()), "lat_sx": (np.uint8, ()), "lat_sy": (np.uint8, ()),
    "lat_ctrl": (np.uint8, ()), "snap_sx_start": (np.uint8, ()), "snap_sy_start": (np.uint8, ()),
    "snap_ctrl_start": (np.uint8, ()), "snap_sx_end": (np.uint8, ()), "snap_sy_end": (np.uint8, ()),
    "snap_ctrl_end": (np.uint8, ()), "snap_mask": (np.uint8, ()), "ctrl_shift": (np.uint8, ()),
    "ctrl_count": (np.uint8, ()), "ctrl_strobe": (np.uint8, ()), "prev_x": (np.int32, ()),
    "prev_time": (np.int32, ()), "pending_dma": (np.uint32, ()), "episode": (np.uint32, ()),
    "status": (np.uint32, ()), "stat_instructions": (np.uint64, ()), "stat_frames": (np.uint32, ()),
    "stat_budget_hits": (np.uint32, ()), "frames_rgb": (np.uint8, (240, 256, 3)),
    "frames_index": (np.uint8, (240, 256)), "obs_gray84": (np.uint8, (84, 84)),
    "prg_bank": (np.uint8, ()), "chr_bank": (np.uint8, ()), "snap_chr_bank": (np.uint8, ()),
}

_lib = None


def load(path: Path | str | None = None):
    """Load (once) and return the product library; raises if it is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(f"{p} is not built; run `python -m nesle_b200.build` (needs nvcc)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


class NesleError(RuntimeError):
    pass


def check(rc: int, lib=None) -> None:
    if rc == NESLE_OK:
        return
    lib = lib or load()
    msg = lib.nesle_last_error().decode()
    if rc == NESLE_ERR_INVALID:
        raise ValueError(msg)
    raise RuntimeError(msg)


def make_create_args(num_envs: int, frameskip: int, rom: bytes, snapshots=(), env_to_level=None,
                     done_mode: int = DONE_SMB, done_args=(0, 0), seed: int = 0, env_offset: int = 0,
                     device: int = 0, max_instructions_per_frame: int = 0):
    """Build a CreateArgs; returns (args, keepalive) -- keep both alive during the call."""
    rom_buf = ctypes.create_string_buffer(bytes(rom), len(rom))
    snaps = [bytes(s) for s in snapshots]
    bufs = [ctypes.create_string_buffer(s, len(s)) for s in snaps]
    ptrs = (_u8p * max(1, len(snaps)))(*[ctypes.cast(b, _u8p) for b in bufs])
    lens = (ctypes.c_size_t * max(1, len(snaps)))(*[len(s) for s in snaps])
    e2l = None
    if env_to_level is not None:
        e2l = np.ascontiguousarray(np.asarray(env_to_level), dtype=np.uint8)
        if e2l.shape != (num_envs,):
            raise ValueError("env_to_level must have shape (num_envs,)")
    args = CreateArgs(device=device, num_envs=num_envs, frameskip=frameskip, rom=ctypes.cast(rom_buf, _u8p),
                      rom_len=len(rom), snapshots=ptrs, snapshot_lens=lens, num_snapshots=len(snaps),
                      env_to_level=e2l.ctypes.data_as(_u8p) if e2l is not None else None,
                      done_mode=done_mode, done_a=done_args[0], done_b=done_args[1], seed=seed,
                      env_offset=env_offset, max_instructions_per_frame=max_instructions_per_frame)
    return args, (rom_buf, bufs, ptrs, lens, e2l)
