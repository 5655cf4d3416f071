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
// Mapping: one 128-thread block per env. The env's VRAM (8 KiB), OAM and LCD
// registers are staged in shared memory with 16-byte coalesced loads (every
// byte the renderer can touch lies in them). Each output row first resolves
// its sprites into a line of 80 sampled positions (at most 10 sprites x 4
// samples), so a pixel costs one BG fetch and one line read instead of a
// scan of the row's sprites. The image is staged in shared memory so the
// global store is contiguous 16-byte chunks. HBM traffic per env is the
// staged 8.4 KiB read plus the image write.
#include <cuda_runtime.h>
#include <stdint.h>

#include "gbx_layout.h"

namespace gbx {

constexpr int RENDER_THREADS = 128;
constexpr int MAX_SPR = 10;
constexpr int OUT_ROWS = 72;

// scaled (packed renders only, may be null): the same image as the policy
// input a consumer builds from the packed bytes (unpack, to bf16, / 3.0), one
// bf16 per output pixel, as [N][72][80] (s2d = 0) or space-to-depth
// [N][36][40][4] (s2d = 1: pixel (oy, ox) at (oy/2, ox/2, (oy&1)*2 + (ox&1)));
// scale_tab holds
// the bf16 bits of shade / 3 for shades 0..3 (16 bits each).
template <bool PACKED>
__global__ void __launch_bounds__(RENDER_THREADS) render_kernel(DevState st, uint8_t* __restrict__ out,
                                                               int64_t base_offset, int vec,
                                                               uint16_t* __restrict__ scaled, uint64_t scale_tab,
                                                               int s2d) {
  constexpr int BPR = PACKED ? 20 : 80;  // output bytes per row
  constexpr int ENV_BYTES = OUT_ROWS * BPR;
  __shared__ __align__(16) uint8_t vram[0x2000];
  __shared__ __align__(16) uint8_t oam[160];
  __shared__ __align__(16) uint8_t io[16];            // FF40-FF4F
  // winning sprite pixel of each sampled position: left+8 | colour << 8 |
  // palette << 10 | BG priority << 11, 0 = none
  __shared__ __align__(16) uint16_t line[OUT_ROWS][80];
  __shared__ __align__(16) uint8_t img[ENV_BYTES];

  const int env = blockIdx.x;
  const int t = threadIdx.x;
  const uint8_t* m = st.mem + (size_t)env * MEM_SIZE;
  {
    const uint4* src = reinterpret_cast<const uint4*>(m + 0x8000);
    uint4* dst = reinterpret_cast<uint4*>(vram);
#pragma unroll 4
    for (int k = t; k < 0x2000 / 16; k += RENDER_THREADS) dst[k] = src[k];
    if (t < 10) reinterpret_cast<uint4*>(oam)[t] = reinterpret_cast<const uint4*>(m + 0xFE00)[t];
    if (t == 10) *reinterpret_cast<uint4*>(io) = *reinterpret_cast<const uint4*>(m + 0xFF40);
  }
  {
    uint4* l4 = reinterpret_cast<uint4*>(&line[0][0]);
    for (int k = t; k < (int)(sizeof(line) / 16); k += RENDER_THREADS) l4[k] = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  const int lcdc = io[0x0], scy = io[0x2], scx = io[0x3], bgp = io[0x7];
  const int obp0 = io[0x8], obp1 = io[0x9], wy = io[0xA], wx = io[0xB];
  const int sh = (lcdc & 4) ? 16 : 8;

  // sprite line of each output row y = 2*oy: the row's first 10 sprites in
  // OAM order (the count ignores X); at each sampled x (even) the opaque
  // pixel of the sprite with the smallest X wins, ties to the lower OAM index
  if (t < OUT_ROWS) {
    uint16_t* L = line[t];
    if (lcdc & 2) {
      const int y = t * 2;
      int nspr = 0;
      for (int s = 0; s < 40 && nspr < MAX_SPR; s++) {
        const int sy = oam[4 * s], sx = oam[4 * s + 1];
        if (sx == 0 || sy == 0 || sx >= 168 || sy >= 160) continue;
        const int top = sy - 16;
        if (y < top || y >= top + sh) continue;
        nspr++;
        int tile = oam[4 * s + 2];
        const int attr = oam[4 * s + 3];
        int row = y - top;
        if ((attr >> 6) & 1) row = sh - 1 - row;
        if (sh == 16) { tile &= 0xFE; if (row >= 8) { tile++; row -= 8; } }
        const int lo = vram[tile * 16 + row * 2], hi = vram[tile * 16 + row * 2 + 1];
        const int left = sx - 8;
        for (int x = left + (left & 1); x < left + 8; x += 2) {  // the four even x the sprite covers
          if (x < 0 || x >= 160) continue;
          const int pxo = x - left;
          const int bit = ((attr >> 5) & 1) ? pxo : 7 - pxo;
          const int color = (((hi >> bit) & 1) << 1) | ((lo >> bit) & 1);
          if (color == 0) continue;
          const int cur = L[x >> 1];
          if (cur == 0 || left < (cur & 0xFF) - 8)
            L[x >> 1] = (uint16_t)((left + 8) | (color << 8) | (((attr >> 4) & 1) << 10) | (((attr >> 7) & 1) << 11));
        }
      }
    }
  }
  __syncthreads();

  for (int i = t; i < ENV_BYTES; i += RENDER_THREADS) {
    const int oy = i / BPR, ob = i - oy * BPR;
    const int y = oy * 2;
    const bool win_row = (lcdc & 0x20) && y >= wy;
    int packed = 0;
#pragma unroll
    for (int k = 0; k < (PACKED ? 4 : 1); k++) {
      const int ox = PACKED ? ob * 4 + k : ob;
      const int x = ox * 2;
      int shade = 0, bg_color = 0;
      if (lcdc & 1) {
        int px, py, map;
        if (win_row && x >= wx - 7) {
          px = x - (wx - 7); py = y - wy; map = (lcdc & 0x40) ? 0x1C00 : 0x1800;
        } else {
          px = (x + scx) & 0xFF; py = (y + scy) & 0xFF; map = (lcdc & 0x08) ? 0x1C00 : 0x1800;
        }
        const int tid = vram[map + ((py & 0xFF) >> 3) * 32 + ((px & 0xFF) >> 3)];
        int ta = (lcdc & 0x10) ? tid * 16 : 0x1000 + (tid >= 128 ? tid - 256 : tid) * 16;
        ta += (py & 7) * 2;
        const int bit = 7 - (px & 7);
        bg_color = (((vram[ta + 1] >> bit) & 1) << 1) | ((vram[ta] >> bit) & 1);
        shade = (bgp >> (bg_color * 2)) & 3;
      }
      const int e = line[oy][ox];
      if (e) {
        const int color = (e >> 8) & 3;
        if (!(((e >> 11) & 1) && bg_color != 0))
          shade = ((((e >> 10) & 1) ? obp1 : obp0) >> (color * 2)) & 3;
      }
      packed |= (shade & 3) << (2 * k);
    }
    img[i] = (uint8_t)packed;
    if (PACKED && scaled) {
      const uint32_t p0 = (uint32_t)((scale_tab >> (16 * (packed & 3))) & 0xFFFF);
      const uint32_t p1 = (uint32_t)((scale_tab >> (16 * ((packed >> 2) & 3))) & 0xFFFF);
      const uint32_t p2 = (uint32_t)((scale_tab >> (16 * ((packed >> 4) & 3))) & 0xFFFF);
      const uint32_t p3 = (uint32_t)((scale_tab >> (16 * ((packed >> 6) & 3))) & 0xFFFF);
      uint16_t* e = scaled + (size_t)env * (OUT_ROWS * 80);
      if (!s2d) {  // four pixels = one 8-byte store, consecutive threads adjacent
        reinterpret_cast<uint2*>(e)[i] = make_uint2(p0 | (p1 << 16), p2 | (p3 << 16));
      } else {     // pixels (oy, 4ob..4ob+3) -> cells (oy/2, 2ob) and (oy/2, 2ob+1), channels (oy&1)*2 + 0/1
        uint32_t* c = reinterpret_cast<uint32_t*>(e + (((oy >> 1) * 40 + 2 * ob) * 4 + (oy & 1) * 2));
        c[0] = p0 | (p1 << 16);
        c[2] = p2 | (p3 << 16);
      }
    }
  }
  __syncthreads();
  uint8_t* dst = out + base_offset + (int64_t)env * ENV_BYTES;
  if (vec) {
    const uint4* s4 = reinterpret_cast<const uint4*>(img);
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    for (int k = t; k < ENV_BYTES / 16; k += RENDER_THREADS) d4[k] = s4[k];
  } else {
    for (int k = t; k < ENV_BYTES; k += RENDER_THREADS) dst[k] = img[k];
  }
}

// --- env 0's 160x144 frame (kernels/ppu_step.py:11-176) ---------------------
// One block per scanline y, one thread per pixel. The line's registers come
// from the env-0 scanline latches (LCDC, SCX, SCY, BGP, WX, WY, window line,
// OBP0, OBP1 captured when the line started); VRAM and OAM are env 0's
// current memory. The window row is the latched window line counter (the
// downsampled renderer uses y - WY instead). Sprites: the first 10 in OAM
// order that pass the validity and line tests, smallest X then lowest OAM
// index among opaque pixels, OBJ-to-BG priority against the raw BG colour.
__global__ void __launch_bounds__(160) render_bg_env0_kernel(DevState st, uint8_t* __restrict__ out) {
  __shared__ uint8_t oam[160];
  __shared__ uint32_t spr[MAX_SPR];  // left+8 | lo<<8 | hi<<16 | attr<<24, OAM order
  __shared__ int nspr_s;
  const int y = blockIdx.x, x = threadIdx.x;
  const uint8_t* m = st.mem;  // env 0
  const uint8_t* L = st.latch;
  const int lcdc = L[0 * SCREEN_H + y], scx = L[1 * SCREEN_H + y], scy = L[2 * SCREEN_H + y];
  const int bgp = L[3 * SCREEN_H + y], wx = L[4 * SCREEN_H + y], wy = L[5 * SCREEN_H + y];
  const int win_line = L[6 * SCREEN_H + y], obp0 = L[7 * SCREEN_H + y], obp1 = L[8 * SCREEN_H + y];
  oam[x] = m[0xFE00 + x];
  __syncthreads();
  if (x == 0) {
    int n = 0;
    if (lcdc & 2) {
      const int sh = (lcdc & 4) ? 16 : 8;
      for (int k = 0; k < 40 && n < MAX_SPR; k++) {
        const int sy = oam[4 * k], sx = oam[4 * k + 1];
        if (sx == 0 || sy == 0 || sx >= 168 || sy >= 160) continue;
        const int top = sy - 16;
        if (y < top || y >= top + sh) continue;
        int tile = oam[4 * k + 2];
        const int attr = oam[4 * k + 3];
        int row = y - top;
        if ((attr >> 6) & 1) row = sh - 1 - row;
        if (sh == 16) { tile &= 0xFE; if (row >= 8) { tile++; row -= 8; } }
        const int ta = 0x8000 + tile * 16 + row * 2;
        spr[n++] = (uint32_t)sx | ((uint32_t)m[ta] << 8) | ((uint32_t)m[ta + 1] << 16) | ((uint32_t)attr << 24);
      }
    }
    nspr_s = n;
  }
  __syncthreads();
  int shade = 0, bg_color = 0;
  if (lcdc & 1) {
    int px, py, map;
    if ((lcdc & 0x20) && y >= wy && x >= wx - 7) {
      px = x - (wx - 7); py = win_line; map = (lcdc & 0x40) ? 0x9C00 : 0x9800;
    } else {
      px = (x + scx) & 0xFF; py = (y + scy) & 0xFF; map = (lcdc & 0x08) ? 0x9C00 : 0x9800;
    }
    const int tid = m[map + ((py & 0xFF) >> 3) * 32 + ((px & 0xFF) >> 3)];
    int ta = (lcdc & 0x10) ? 0x8000 + tid * 16 : 0x9000 + (tid >= 128 ? tid - 256 : tid) * 16;
    ta += (py & 7) * 2;
    const int bit = 7 - (px & 7);
    bg_color = (((m[ta + 1] >> bit) & 1) << 1) | ((m[ta] >> bit) & 1);
    shade = (bgp >> (bg_color * 2)) & 3;
  }
  int best_left = 1 << 30, best_color = 0, best_attr = 0;
  for (int j = 0; j < nspr_s; j++) {
    const uint32_t e = spr[j];
    const int left = (int)(e & 0xFF) - 8;
    if (x < left || x >= left + 8 || left >= best_left) continue;
    const int attr = e >> 24, lo = (e >> 8) & 0xFF, hi = (e >> 16) & 0xFF;
    const int pxo = x - left;
    const int bit = ((attr >> 5) & 1) ? pxo : 7 - pxo;
    const int color = (((hi >> bit) & 1) << 1) | ((lo >> bit) & 1);
    if (color == 0) continue;
    best_left = left; best_color = color; best_attr = attr;
  }
  if (best_color && !(((best_attr >> 7) & 1) && bg_color != 0))
    shade = ((((best_attr >> 4) & 1) ? obp1 : obp0) >> (best_color * 2)) & 3;
  out[y * 160 + x] = (uint8_t)shade;
}

cudaError_t launch_render_bg_env0(const DevState& st, uint8_t* out, cudaStream_t stream) {
  render_bg_env0_kernel<<<SCREEN_H, 160, 0, stream>>>(st, out);
  return cudaGetLastError();
}

cudaError_t launch_render(const DevState& st, uint8_t* out, int64_t base_offset, bool packed,
                          cudaStream_t stream, uint16_t* scaled, uint64_t scale_tab, int s2d) {
  // every env image starts 16-byte aligned when the buffer start is (1440 and 5760 are multiples of 16)
  const int vec = ((reinterpret_cast<uintptr_t>(out) + (uintptr_t)base_offset) & 15) == 0;
  if (packed)
    render_kernel<true><<<st.n, RENDER_THREADS, 0, stream>>>(st, out, base_offset, vec, scaled, scale_tab, s2d);
  else
    render_kernel<false><<<st.n, RENDER_THREADS, 0, stream>>>(st, out, base_offset, vec, nullptr, 0, 0);
  return cudaGetLastError();
}

}  // namespace gbx
