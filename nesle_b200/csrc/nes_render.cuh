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

// CHR byte at pattern address a (< $2000): CHR mirrored over its size, 0
// without CHR ROM.  Power-of-two sizes (8 KB for NROM) skip the division.
NESLE_HD uint32_t rv_chr(const RenderView& v, uint32_t a) {
    if (!v.chr_size) return 0u;
    return v.chr[(v.chr_size & (v.chr_size - 1u)) ? a % v.chr_size : a & (v.chr_size - 1u)];
}
NESLE_HD uint32_t rv_mem(const RenderView& v, uint32_t a) {  // batch_render.cuh:104-121
    a &= 0x3FFF;
    if (a < 0x2000) return rv_chr(v, a);
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
// Background tile of row y at scrolled column wx (batch_render.cuh:161-204):
// its pattern row (bits 0-15: low plane, high plane) and palette group (bits
// 16-17).  Every pixel of the row inside that tile shares the entry.
NESLE_HD uint32_t rv_tile_entry(const RenderView& v, uint32_t y, uint32_t wx) {
    const uint32_t wy = v.sy + y, cy = (wy % 240) / 8, fy = wy & 7;
    const uint32_t base = v.ctrl & 3;
    const uint32_t nty = ((base >> 1) + wy / 240) & 1;
    const uint32_t cx = (wx & 0xFF) / 8;
    const uint32_t ntx = ((base & 1) + wx / 256) & 1;
    const uint32_t ntb = 0x2000 + (ntx | (nty << 1)) * 0x400;
    const uint32_t pb = (v.ctrl & 0x10) ? 0x1000 : 0;
    // Every address here is nametable space below $3000 or pattern space below
    // $2000, so rv_mem's range dispatch reduces to these two reads.
    const uint32_t tile = v.nt[mirror_nt(v.horizontal, ntb + cy * 32 + cx)];
    const uint32_t lo = rv_chr(v, pb + tile * 16 + fy), hi = rv_chr(v, pb + tile * 16 + fy + 8);
    const uint32_t at = v.nt[mirror_nt(v.horizontal, ntb + 0x3C0 + (cy / 4) * 8 + cx / 4)];
    const uint32_t group = (at >> (((cy & 2) << 1) | (cx & 2))) & 3;
    return lo | (hi << 8) | (group << 16);
}
// Colour index of background pixel x (scrolled column wx) from its tile entry; 0 = transparent.
NESLE_HD uint32_t rv_bg_from_entry(const RenderView& v, uint32_t entry, uint32_t x, uint32_t wx) {
    if (!(v.mask & 0x08) || (!(v.mask & 0x02) && x < 8)) return 0;
    const uint32_t bit = 7 - (wx & 7);
    const uint32_t c = ((entry >> bit) & 1) | (((entry >> (8 + bit)) & 1) << 1);
    if (c == 0) return 0;
    return rv_palette(v, ((entry >> 16) & 3) * 4 + c);
}
NESLE_HD uint32_t rv_background(const RenderView& v, uint32_t x, uint32_t y) {
    const uint32_t wx = v.sx + x;
    return rv_bg_from_entry(v, rv_tile_entry(v, y, wx), x, wx);
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

// The views read the presentation snapshot through the given pointers (global
// rows, or a CTA's shared-memory copy of them).
NESLE_HD RenderEnv render_env_at(const EnvRecord& r, const uint8_t* nt, const uint8_t* pal, const uint8_t* oam,
                                 const uint8_t* chr, uint32_t chr_size, uint32_t horizontal) {
    RenderEnv e;
    RenderView play;
    play.nt = nt;
    play.pal = pal;
    play.oam = oam;
    play.chr = chr;
    play.chr_size = chr_size;
    play.horizontal = horizontal;
    play.sx = r.snap_sx_end; play.sy = r.snap_sy_end; play.ctrl = r.snap_ctrl_end; play.mask = r.snap_mask;
    e.hud = play;
    e.hud.sx = r.snap_sx_start; e.hud.sy = r.snap_sy_start; e.hud.ctrl = r.snap_ctrl_start;
    int split = (int)play.oam[0] + 1 + ((play.ctrl & 0x20) ? 16 : 8);
    e.lower = play;
    if (split >= 240) { e.lower = e.hud; split = 0; }
    e.split = split;
    return e;
}

// The pattern tables a presentation snapshot renders with: the whole CHR
// ROM, or for CNROM the 8 KB bank latched at vblank.
NESLE_HD const uint8_t* snapshot_chr(const BatchView& bv, uint32_t env, uint32_t& size) {
    if (bv.mapper == kMapperCnrom && bv.chr_size) {
        size = 8192u;
        return bv.chr + (size_t)bv.mstate[env].snap_chr_bank * 8192u;
    }
    size = bv.chr_size;
    return bv.chr;
}

NESLE_HD RenderEnv render_env(const BatchView& bv, const EnvRecord& r, uint32_t env) {
    uint32_t chr_size;
    const uint8_t* chr = snapshot_chr(bv, env, chr_size);
    return render_env_at(r, bv.snap_nt + (size_t)env * kNtBytes, bv.snap_pal + (size_t)env * kPalBytes,
                         bv.snap_oam + (size_t)env * kOamBytes, chr, chr_size, bv.horizontal);
}

// Bit i set when sprite i covers scanline y (the row test of the sprite loop,
// hoisted so a pixel visits only the sprites on its row).
NESLE_HD uint64_t sprite_row_mask(const RenderEnv& e, uint32_t y) {
    const RenderView& s = e.lower;
    const int h = (s.ctrl & 0x20) ? 16 : 8;
    uint64_t m = 0;
    for (uint32_t i = 0; i < 64; ++i) {
        const int sy = (int)y - ((int)s.oam[i * 4] + 1);
        if (sy >= 0 && sy < h) m |= 1ull << i;
    }
    return m;
}

// Bit i set when sprite i overlaps pixel columns 8 g .. 8 g + 7 (a sprite
// covers X .. X + 7); ANDed with the row mask it leaves the sprites a pixel
// can see.
NESLE_HD uint64_t sprite_col_mask(const RenderEnv& e, uint32_t g) {
    uint64_t m = 0;
    for (uint32_t i = 0; i < 64; ++i) {
        const uint32_t x = e.lower.oam[i * 4 + 3];
        if (x <= 8 * g + 7 && x + 7 >= 8 * g) m |= 1ull << i;
    }
    return m;
}

NESLE_HD uint32_t lowest_set(uint64_t m) {
#if defined(__CUDA_ARCH__)
    return (uint32_t)(__ffsll((long long)m) - 1);
#else
    return (uint32_t)__builtin_ctzll(m);
#endif
}

// The view that paints row y's background (two-region split).
NESLE_HD const RenderView& bg_view(const RenderEnv& e, uint32_t y) { return ((int)y < e.split) ? e.hud : e.lower; }

// ---------------------------------------------------------------------------
// Pixel composition, render_batch_rgb_pixel_env (:378-434), from tables: the
// env's 32 palette entries resolved once (`res[i]` = rv_palette(view, i); both
// views share palette and mask), each sprite's pattern rows with flips applied,
// and per-row tile entries of the background.
// ---------------------------------------------------------------------------
NESLE_HD void resolve_palette(const RenderEnv& e, uint8_t* res) {
    for (uint32_t i = 0; i < 32; ++i) res[i] = (uint8_t)rv_palette(e.lower, i);
}

NESLE_HD uint32_t reverse8(uint32_t b) {
#if defined(__CUDA_ARCH__)
    return __brev(b) >> 24;
#else
    b = ((b & 0xF0u) >> 4) | ((b & 0x0Fu) << 4);
    b = ((b & 0xCCu) >> 2) | ((b & 0x33u) << 2);
    return ((b & 0xAAu) >> 1) | ((b & 0x55u) << 1);
#endif
}

// Row r (0..15) of sprite i with any flips applied: pixel sx of the row at
// bit sx of the low (bits 0-7) and high (bits 8-15) plane.  Same pixels as
// rv_sprite_px over sx = 0..7: one pattern byte pair, reversed unless the
// sprite is flipped horizontally (pattern pixel p sits at bit 7 - p).
NESLE_HD uint32_t sprite_pattern_row(const RenderView& s, uint32_t i, uint32_t r) {
    const uint8_t* so = s.oam + i * 4;
    const uint32_t tile = so[1], attr = so[2];
    uint32_t base;
    if (s.ctrl & 0x20) {  // 8x16
        const uint32_t py = (attr & 0x80) ? 15u - r : r;
        base = ((tile & 1u) ? 0x1000u : 0u) + (((tile & 0xFEu) + py / 8u) & 0xFFu) * 16u + (py & 7u);
    } else {
        const uint32_t py = (attr & 0x80) ? 7u - r : r;
        base = ((s.ctrl & 0x08) ? 0x1000u : 0u) + tile * 16u + py;
    }
    uint32_t lo = rv_chr(s, base), hi = rv_chr(s, base + 8u);
    if (!(attr & 0x40)) {
        lo = reverse8(lo);
        hi = reverse8(hi);
    }
    return lo | (hi << 8);
}

// Colour index of pixel (x, y) given its background colour `bgc` (0 =
// transparent, from bg_view): the lowest-index opaque sprite covering it wins,
// a behind-background sprite only over transparent background.
// `spat[i * 16 + r]` is sprite_pattern_row(lower, i, r) and `rows` any superset
// of the sprites covering the pixel (the row mask ANDed with the column mask).
NESLE_HD uint32_t compose_pixel_tables(const RenderEnv& e, const uint8_t* res, uint32_t x, uint32_t y, uint32_t bgc,
                                       uint64_t rows, const uint16_t* spat) {
    const RenderView& s = e.lower;
    uint32_t c = bgc ? bgc : res[0];
    if ((s.mask & 0x10) && ((s.mask & 0x04) || x >= 8)) {
        while (rows) {
            const uint32_t i = lowest_set(rows);
            rows &= rows - 1;
            const uint8_t* so = s.oam + i * 4;
            const uint32_t sx = x - so[3];
            if (sx >= 8) continue;
            const uint32_t pat = spat[i * 16 + (y - so[0] - 1)];
            const uint32_t sc = ((pat >> sx) & 1u) | (((pat >> (8 + sx)) & 1u) << 1);
            if (sc == 0) continue;
            const uint32_t attr = so[2];
            if ((attr & 0x20) && ((int)y >= e.split ? bgc : rv_background(s, x, y)) != 0) continue;
            c = res[0x10 + (attr & 3) * 4 + sc];
            break;
        }
    }
    return c;
}

// Background colour of pixel x from its tile entry and the resolved palette.
NESLE_HD uint32_t bg_from_entry_tables(const RenderView& v, const uint8_t* res, uint32_t entry, uint32_t x, uint32_t wx) {
    if (!(v.mask & 0x08) || (!(v.mask & 0x02) && x < 8)) return 0;
    const uint32_t bit = 7 - (wx & 7);
    const uint32_t c = ((entry >> bit) & 1) | (((entry >> (8 + bit)) & 1) << 1);
    return c ? res[((entry >> 16) & 3) * 4 + c] : 0u;
}

// Tile slots of one row: slot j holds the tile of scrolled column
// (sx & ~7) + 8 j; 256 pixels touch at most 33 of them.
constexpr uint32_t kRowTiles = 33;
NESLE_HD uint32_t tile_slot(const RenderView& v, uint32_t x) { return ((v.sx + x) >> 3) - (v.sx >> 3); }
NESLE_HD uint32_t slot_entry(const RenderView& v, uint32_t y, uint32_t j) {
    return rv_tile_entry(v, y, (v.sx & ~7u) + 8 * j);
}

// 84x84 grey: output (ox, oy) is the integer area average of the luma of the
// source pixels it covers.  In units of 1/21 px horizontally and 1/7 px
// vertically, source column sx spans [21 sx, 21 sx + 21) and output column ox
// [64 ox, 64 ox + 64); source row sy spans [7 sy, 7 sy + 7) and output row oy
// [20 oy, 20 oy + 20).  Result = (sum(luma * wx * wy) + 640) / 1280.  Source
// rows [20 k, 20 k + 20) map exactly onto output rows [7 k, 7 k + 7).
constexpr uint32_t kGrayStripRows = 20, kGrayStripOut = 7;

NESLE_HD uint32_t umin(uint32_t a, uint32_t b) { return a < b ? a : b; }
NESLE_HD uint32_t umax(uint32_t a, uint32_t b) { return a > b ? a : b; }

NESLE_HD uint32_t luma_of_rgb(uint32_t r, uint32_t g, uint32_t b) {  // BT.601, rounded
    return (299u * r + 587u * g + 114u * b + 500u) / 1000u;
}

// One output pixel from a strip of source luma (`luma[row * 256 + x]`, rows
// relative to `row0`).
NESLE_HD uint32_t gray84_pixel(const uint8_t* luma, uint32_t row0, uint32_t ox, uint32_t oy) {
    uint32_t acc = 0;
    for (uint32_t sy = (20 * oy) / 7; sy <= (20 * oy + 19) / 7; ++sy) {
        const uint32_t wy = umin(7 * sy + 7, 20 * oy + 20) - umax(7 * sy, 20 * oy);
        for (uint32_t sx = (64 * ox) / 21; sx <= (64 * ox + 63) / 21; ++sx) {
            const uint32_t wx = umin(21 * sx + 21, 64 * ox + 64) - umax(21 * sx, 64 * ox);
            acc += luma[(sy - row0) * kFrameW + sx] * wx * wy;
        }
    }
    return (acc + 640) / 1280;
}

}  // namespace nesle
