// nes_render.cuh -- per-pixel renderer over the vblank presentation snapshot.
//
// Restates cpp/include/nesle/cuda/batch_render.cuh:104-434: background from the
// snapshot nametables with the two-region scroll split at sprite 0's bottom
// edge (resolve_render_env_views, :333-370), then the lowest-index opaque,
// un-occluded sprite (render_batch_rgb_pixel_env, :378-434).  The product of a
// pixel is its NES colour index (0-63); RGB is a table lookup and the 84x84
// grey observation an exact integer area resample of the luma of those
// indices (this build's addition, no counterpart in the reference).
#pragma once
#include "nes_core.cuh"

namespace nesle {

// 2C02 palette as in batch_render.cuh:23-40.
#define NESLE_PALETTE_RGB                                                                  \
    {0x54, 0x54, 0x54, 0x00, 0x1e, 0x74, 0x08, 0x10, 0x90, 0x30, 0x00, 0x88, 0x44, 0x00, 0x64, \
     0x5c, 0x00, 0x30, 0x54, 0x04, 0x00, 0x3c, 0x18, 0x00, 0x20, 0x2a, 0x00, 0x08, 0x3a, 0x00, \
     0x00, 0x40, 0x00, 0x00, 0x3c, 0x00, 0x00, 0x32, 0x3c, 0x00, 0x00, 0x00, 0x00, 0x00, 0x00, \
     0x00, 0x00, 0x00, 0x98, 0x96, 0x98, 0x08, 0x4c, 0xc4, 0x30, 0x32, 0xec, 0x5c, 0x1e, 0xe4, \
     0x88, 0x14, 0xb0, 0xa0, 0x14, 0x64, 0x98, 0x22, 0x20, 0x78, 0x3c, 0x00, 0x54, 0x5a, 0x00, \
     0x28, 0x72, 0x00, 0x08, 0x7c, 0x00, 0x00, 0x76, 0x28, 0x00, 0x66, 0x78, 0x00, 0x00, 0x00, \
     0x00, 0x00, 0x00, 0x00, 0x00, 0x00, 0xec, 0xee, 0xec, 0x4c, 0x9a, 0xec, 0x78, 0x7c, 0xec, \
     0xb0, 0x62, 0xec, 0xe4, 0x54, 0xec, 0xec, 0x58, 0xb4, 0xec, 0x6a, 0x64, 0xd4, 0x88, 0x20, \
     0xa0, 0xaa, 0x00, 0x74, 0xc4, 0x00, 0x4c, 0xd0, 0x20, 0x38, 0xcc, 0x6c, 0x38, 0xb4, 0xcc, \
     0x3c, 0x3c, 0x3c, 0x00, 0x00, 0x00, 0x00, 0x00, 0x00, 0xec, 0xee, 0xec, 0xa8, 0xcc, 0xec, \
     0xbc, 0xbc, 0xec, 0xd4, 0xb2, 0xec, 0xec, 0xae, 0xec, 0xec, 0xae, 0xd4, 0xec, 0xb4, 0xb0, \
     0xe4, 0xc4, 0x90, 0xcc, 0xd2, 0x78, 0xb4, 0xde, 0x78, 0xa8, 0xe2, 0x90, 0x98, 0xe2, 0xb4, \
     0xa0, 0xd6, 0xe4, 0xa0, 0xa2, 0xa0, 0x00, 0x00, 0x00, 0x00, 0x00, 0x00}

// One view of the presentation snapshot (scroll/ctrl/mask + memories).
struct RenderView {
    const uint8_t* nt;
    const uint8_t* pal;
    const uint8_t* oam;
    const uint8_t* chr;
    uint32_t chr_size, horizontal;
    uint32_t sx, sy, ctrl, mask;
};

NESLE_HD uint32_t rv_mem(const RenderView& v, uint32_t a) {  // batch_render.cuh:104-121
    a &= 0x3FFF;
    if (a < 0x2000) return v.chr_size ? v.chr[a % v.chr_size] : 0u;
    if (a < 0x3F00) {
        if (a >= 0x3000) a -= 0x1000;
        return v.nt[mirror_nt(v.horizontal, a)];
    }
    return v.pal[mirror_pal(a)];
}
NESLE_HD uint32_t rv_palette(const RenderView& v, uint32_t idx) {  // :123-131
    uint32_t c = rv_mem(v, 0x3F00 + idx);
    if (v.mask & 1) c &= 0x30;
    return c & 0x3F;
}
NESLE_HD uint32_t rv_pattern(const RenderView& v, uint32_t tile_base, uint32_t fx, uint32_t fy) {  // :148-159
    const uint32_t lo = rv_mem(v, tile_base + fy), hi = rv_mem(v, tile_base + fy + 8);
    const uint32_t bit = 7 - fx;
    return ((lo >> bit) & 1) | (((hi >> bit) & 1) << 1);
}
NESLE_HD uint32_t rv_background(const RenderView& v, uint32_t x, uint32_t y) {  // :161-204
    if (!(v.mask & 0x08) || (!(v.mask & 0x02) && x < 8)) return 0;
    const uint32_t wy = v.sy + y, cy = (wy % 240) / 8, fy = wy & 7;
    const uint32_t base = v.ctrl & 3;
    const uint32_t nty = ((base >> 1) + wy / 240) & 1;
    const uint32_t wx = v.sx + x, cx = (wx & 0xFF) / 8, fx = wx & 7;
    const uint32_t ntx = ((base & 1) + wx / 256) & 1;
    const uint32_t ntb = 0x2000 + (ntx | (nty << 1)) * 0x400;
    const uint32_t pb = (v.ctrl & 0x10) ? 0x1000 : 0;
    const uint32_t tile = rv_mem(v, ntb + cy * 32 + cx);
    const uint32_t c = rv_pattern(v, pb + tile * 16, fx, fy);
    if (c == 0) return 0;
    const uint32_t at = rv_mem(v, ntb + 0x3C0 + (cy / 4) * 8 + cx / 4);
    const uint32_t shift = ((cy & 2) << 1) | (cx & 2);
    return rv_palette(v, ((at >> shift) & 3) * 4 + c);
}
NESLE_HD uint32_t rv_sprite_px(const RenderView& v, uint32_t tile, uint32_t attr, uint32_t px, uint32_t py) {  // :206-240
    if (attr & 0x40) px = 7 - px;
    if (v.ctrl & 0x20) {
        if (attr & 0x80) py = 15 - py;
        const uint32_t pb = (tile & 1) ? 0x1000 : 0;
        const uint32_t tn = ((tile & 0xFE) + py / 8) & 0xFF;
        return rv_pattern(v, pb + tn * 16, px, py & 7);
    }
    if (attr & 0x80) py = 7 - py;
    const uint32_t pb = (v.ctrl & 0x08) ? 0x1000 : 0;
    return rv_pattern(v, pb + tile * 16, px, py);
}

// The two views and split row of one env (resolve_render_env_views).
struct RenderEnv {
    RenderView hud, lower;
    int split;
};

NESLE_HD RenderEnv render_env(const BatchView& bv, const EnvRecord& r, uint32_t env) {
    RenderEnv e;
    RenderView play;
    play.nt = bv.snap_nt + (size_t)env * kNtBytes;
    play.pal = bv.snap_pal + (size_t)env * kPalBytes;
    play.oam = bv.snap_oam + (size_t)env * kOamBytes;
    play.chr = bv.chr;
    play.chr_size = bv.chr_size;
    play.horizontal = bv.horizontal;
    play.sx = r.snap_sx_end; play.sy = r.snap_sy_end; play.ctrl = r.snap_ctrl_end; play.mask = r.snap_mask;
    e.hud = play;
    e.hud.sx = r.snap_sx_start; e.hud.sy = r.snap_sy_start; e.hud.ctrl = r.snap_ctrl_start;
    int split = (int)play.oam[0] + 1 + ((play.ctrl & 0x20) ? 16 : 8);
    e.lower = play;
    if (split >= 240) { e.lower = e.hud; split = 0; }
    e.split = split;
    return e;
}

// render_batch_rgb_pixel_env (:378-434), returning the colour index.
NESLE_HD uint32_t render_pixel(const RenderEnv& e, uint32_t x, uint32_t y) {
    const RenderView& bg = ((int)y < e.split) ? e.hud : e.lower;
    const RenderView& s = e.lower;
    uint32_t c = rv_background(bg, x, y);
    if (c == 0) c = rv_palette(s, 0);
    if ((s.mask & 0x10) && ((s.mask & 0x04) || x >= 8)) {
        const uint32_t h = (s.ctrl & 0x20) ? 16 : 8;
        for (uint32_t i = 0; i < 64; ++i) {
            const uint8_t* so = s.oam + i * 4;
            const int sy = (int)y - ((int)so[0] + 1);
            if (sy < 0 || sy >= (int)h) continue;
            const int sx = (int)x - (int)so[3];
            if (sx < 0 || sx >= 8) continue;
            const uint32_t attr = so[2];
            if ((attr & 0x20) && rv_background(s, x, y) != 0) continue;
            const uint32_t sc = rv_sprite_px(s, so[1], attr, (uint32_t)sx, (uint32_t)sy);
            if (sc == 0) continue;
            c = rv_palette(s, 0x10 + (attr & 3) * 4 + sc);
            break;
        }
    }
    return c;
}

}  // namespace nesle
