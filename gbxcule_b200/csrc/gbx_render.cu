// gbx_render.cu - snapshot renderer: downsampled 72x80 shades of every env's
// current memory, packed 2 bpp (72x20 bytes) or one byte per pixel.
//
// Output is bit-identical to the reference's
// ppu_render_shades_downsampled_{packed_,}all_envs
// (src/gbxcule/kernels/ppu_render_downsampled.py:27-234): the top-left pixel
// of each 2x2 block; BG or window (window row = y - WY); LCDC.0 off gives BG
// shade 0 but sprites still draw; sprites are the first 10 in OAM order that
// pass the validity and line tests (the count ignores X), the winner is the
// opaque sprite with the smallest X and then the lowest OAM index, and
// OBJ-to-BG priority compares against the raw BG colour.
//
// Mapping: lane = env, so every IO/OAM/VRAM read of a warp is one address
// across 32 consecutive envs (one sector in the interleaved layout). A warp
// renders a group of rows for its 32 envs. OAM is staged in shared memory once,
// each row builds its sprite line list once (not 40 OAM reads per pixel), BG
// tile rows are reused across the four samples that fall in one tile, and
// output rows are staged in shared memory so global stores are contiguous
// 16-byte chunks.
#include <cuda_runtime.h>
#include <stdint.h>

#include "gbx_layout.h"

namespace gbx {

constexpr int RW_WARPS = 4;            // warps per block
constexpr int MAX_SPR = 10;

struct RenderSmem {
  uint8_t oam[RW_WARPS][160][32];      // [warp][byte][lane]
  uint32_t spr[RW_WARPS][MAX_SPR][32]; // line list: left | lo<<8 | hi<<16 | attr<<24
  uint8_t out[RW_WARPS][32][80];       // staged output rows
};

template <bool PACKED, bool VEC>
__global__ void __launch_bounds__(RW_WARPS * 32) render_kernel(DevState st, uint8_t* __restrict__ out,
                                                              int64_t base_offset) {
  __shared__ __align__(16) RenderSmem sm;
  constexpr int ROWS = PACKED ? 4 : 1;              // output rows per task
  constexpr int GROUPS = 72 / ROWS;
  constexpr int ENV_BYTES = PACKED ? PACKED_BYTES : SHADE_BYTES;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int task = blockIdx.x * RW_WARPS + warp;
  const int env_groups = (st.n + 31) >> 5;
  if (task >= env_groups * GROUPS) return;
  const int eg = task / GROUPS, rg = task - eg * GROUPS;
  const int env0 = eg * 32, env = env0 + lane;
  const bool live = env < st.n;
  const size_t S = (size_t)st.S;
  const uint8_t* m = st.mem + (live ? env : env0);
  auto M = [&](int a) -> int { return m[(size_t)a * S]; };

  const int lcdc = M(0xFF40), scy = M(0xFF42), scx = M(0xFF43), bgp = M(0xFF47);
  const int obp0 = M(0xFF48), obp1 = M(0xFF49), wy = M(0xFF4A), wx = M(0xFF4B);
  const bool obj_on = lcdc & 2;
  const int sh = (lcdc & 4) ? 16 : 8;
  if (obj_on) {
#pragma unroll 4
    for (int b = 0; b < 160; b++) sm.oam[warp][b][lane] = (uint8_t)M(0xFE00 + b);
  }

  for (int r = 0; r < ROWS; r++) {
    const int oy = rg * ROWS + r;
    const int y = oy * 2;
    // sprite line list for this row (first 10 in OAM order)
    int nspr = 0;
    if (obj_on) {
      for (int s = 0; s < 40 && nspr < MAX_SPR; s++) {
        int sy = sm.oam[warp][4 * s][lane], sx = sm.oam[warp][4 * s + 1][lane];
        if (sx == 0 || sy == 0 || sx >= 168 || sy >= 160) continue;
        int top = sy - 16;
        if (y < top || y >= top + sh) continue;
        int tile = sm.oam[warp][4 * s + 2][lane], attr = sm.oam[warp][4 * s + 3][lane];
        int row = y - top;
        if ((attr >> 6) & 1) row = sh - 1 - row;
        if (sh == 16) { tile &= 0xFE; if (row >= 8) { tile++; row -= 8; } }
        int ta = 0x8000 + tile * 16 + row * 2;
        int lo = M(ta), hi = M(ta + 1);
        sm.spr[warp][nspr][lane] = (uint32_t)(sx - 8 + 8) | (lo << 8) | (hi << 16) | (attr << 24);
        nspr++;
      }
    }
    // BG/window tile cache
    int cached_tile = -1, tlo = 0, thi = 0;
    const bool win_row = (lcdc & 0x20) && y >= wy;
    for (int ob = 0; ob < (PACKED ? 20 : 80); ob++) {
      int packed = 0;
#pragma unroll
      for (int k = 0; k < (PACKED ? 4 : 1); k++) {
        const int x = PACKED ? (ob * 4 + k) * 2 : ob * 2;
        int shade = 0, bg_color = 0;
        if (lcdc & 1) {
          int px, py, map;
          if (win_row && x >= wx - 7) {
            px = x - (wx - 7); py = y - wy; map = (lcdc & 0x40) ? 0x9C00 : 0x9800;
          } else {
            px = (x + scx) & 0xFF; py = (y + scy) & 0xFF; map = (lcdc & 0x08) ? 0x9C00 : 0x9800;
          }
          int map_addr = map + ((py & 0xFF) >> 3) * 32 + ((px & 0xFF) >> 3);
          int key = (map_addr << 3) | (py & 7);
          if (key != cached_tile) {
            int tid = M(map_addr);
            int ta = (lcdc & 0x10) ? 0x8000 + tid * 16 : 0x9000 + (tid >= 128 ? tid - 256 : tid) * 16;
            ta += (py & 7) * 2;
            tlo = M(ta); thi = M(ta + 1);
            cached_tile = key;
          }
          int bit = 7 - (px & 7);
          bg_color = (((thi >> bit) & 1) << 1) | ((tlo >> bit) & 1);
          shade = (bgp >> (bg_color * 2)) & 3;
        }
        if (nspr) {
          int best_left = 1 << 30, best_color = 0, best_attr = 0;
          for (int j = 0; j < nspr; j++) {
            uint32_t e = sm.spr[warp][j][lane];
            int left = (int)(e & 0xFF) - 8;
            if (x < left || x >= left + 8 || left >= best_left) continue;
            int attr = e >> 24, lo = (e >> 8) & 0xFF, hi = (e >> 16) & 0xFF;
            int pxo = x - left;
            int bit = ((attr >> 5) & 1) ? pxo : 7 - pxo;
            int color = (((hi >> bit) & 1) << 1) | ((lo >> bit) & 1);
            if (color == 0) continue;
            best_left = left; best_color = color; best_attr = attr;
          }
          if (best_color && !(((best_attr >> 7) & 1) && bg_color != 0)) {
            int pal = ((best_attr >> 4) & 1) ? obp1 : obp0;
            shade = (pal >> (best_color * 2)) & 3;
          }
        }
        packed |= (shade & 3) << (2 * k);
      }
      sm.out[warp][lane][r * (PACKED ? 20 : 80) + ob] = (uint8_t)packed;
    }
  }
  __syncwarp();
  // cooperative store: 32 envs x 80 bytes (5 chunks of 16 B per env)
  const int64_t row_off = (int64_t)rg * 80;
  if (VEC) {
    for (int c = lane; c < 32 * 5; c += 32) {
      int el = c / 5, part = c - el * 5;
      if (env0 + el >= st.n) continue;
      uint4 v = *reinterpret_cast<const uint4*>(&sm.out[warp][el][part * 16]);
      *reinterpret_cast<uint4*>(out + base_offset + (int64_t)(env0 + el) * ENV_BYTES + row_off + part * 16) = v;
    }
  } else {
    for (int c = lane; c < 32 * 80; c += 32) {
      int el = c / 80, b = c - el * 80;
      if (env0 + el >= st.n) continue;
      out[base_offset + (int64_t)(env0 + el) * ENV_BYTES + row_off + b] = sm.out[warp][el][b];
    }
  }
}

cudaError_t launch_render(const DevState& st, uint8_t* out, int64_t base_offset, bool packed,
                          cudaStream_t stream) {
  const int groups = packed ? 18 : 72;
  const int tasks = ((st.n + 31) / 32) * groups;
  const int blocks = (tasks + RW_WARPS - 1) / RW_WARPS;
  const bool vec = ((reinterpret_cast<uintptr_t>(out) + (uintptr_t)base_offset) & 15) == 0;
  if (packed) {
    if (vec) render_kernel<true, true><<<blocks, RW_WARPS * 32, 0, stream>>>(st, out, base_offset);
    else render_kernel<true, false><<<blocks, RW_WARPS * 32, 0, stream>>>(st, out, base_offset);
  } else {
    if (vec) render_kernel<false, true><<<blocks, RW_WARPS * 32, 0, stream>>>(st, out, base_offset);
    else render_kernel<false, false><<<blocks, RW_WARPS * 32, 0, stream>>>(st, out, base_offset);
  }
  return cudaGetLastError();
}

}  // namespace gbx
