// gbx_state.cu - whole-state kernels: initial state, snapshot capture, masked
// restore, and conversion to the reference's env-major layout.
//
// The masked restore replaces the reference's ~37 launches of
// reset_copy_{strided,scalar}_* (src/gbxcule/kernels/reset_mask.py:12-79,
// driven by src/gbxcule/core/reset_cache.py:192-307) with one launch. It
// restores exactly the fields ResetCache restores: the 64 KiB address space,
// cart_state, cart RAM, the serial buffer and every per-env scalar, including
// the host-path action buffer; env-0 latches, obs and reward are untouched.
// Work item = (4-env column, chunk of 256 address rows): the mask is read once
// per item, items whose four envs are all unmasked return at once, and the
// others do a coalesced 4-byte read-merge-write per row.
#include <cuda_runtime.h>
#include <stdint.h>

#include "gbx_layout.h"

namespace gbx {



constexpr int ROW_CHUNK = 256;

// --- initial state (src/gbxcule/backends/warp_vec.py:249-497) ---------------
// Expects every buffer zeroed beforehand.
__global__ void init_kernel(DevState st) {
  const size_t S = (size_t)st.S;
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  const int stride = gridDim.x * blockDim.x;
  // boot ROM bytes at 0x0000-0x00FF of every env
  for (int k = tid; k < 256 * st.S; k += stride) {
    int a = k / st.S, e = k - a * st.S;
    if (e < st.n) st.mem[(size_t)a * S + e] = st.boot[a];
  }
  for (int e = tid; e < st.n; e += stride) {
    st.cart_state[(size_t)CS_MBC_KIND * S + e] = st.mbc_kind;
    st.cart_state[(size_t)CS_ROM_BANK_LO * S + e] = 1;
    st.cart_state[(size_t)CS_BOOTROM * S + e] = 1;
    st.u8s[(size_t)F_JOYP_SELECT * S + e] = 0x30;
  }
}

// --- snapshot capture (reset_cache.py:67-190) ----------------------------------
__global__ void snapshot_kernel(DevState st, Snapshot snap, int env) {
  const size_t S = (size_t)st.S;
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  const int stride = gridDim.x * blockDim.x;
  for (int a = tid; a < MEM_SIZE; a += stride) snap.mem[a] = st.mem[(size_t)a * S + env];
  for (int a = tid; a < snap.ram_bytes; a += stride) snap.cart_ram[a] = st.cart_ram[(size_t)a * S + env];
  for (int a = tid; a < SERIAL_MAX; a += stride) snap.serial[a] = st.serial[(size_t)a * S + env];
  if (tid < CS_STRIDE) snap.cart_state[tid] = st.cart_state[(size_t)tid * S + env];
  if (tid < I32_COUNT) snap.i32[tid] = st.i32[(size_t)tid * S + env];
  if (tid < I64_COUNT) snap.i64[tid] = st.i64[(size_t)tid * S + env];
  if (tid < U8_COUNT) snap.u8s[tid] = st.u8s[(size_t)tid * S + env];
}

// --- masked restore --------------------------------------------------------------
__device__ __forceinline__ uint32_t mask4(const uint8_t* mask, int n, int e0) {
  uint32_t m = 0;
#pragma unroll
  for (int k = 0; k < 4; k++)
    if (e0 + k < n && mask[e0 + k]) m |= 0xFFu << (8 * k);
  return m;
}

__device__ __forceinline__ void restore_rows(uint8_t* base, const uint8_t* src, int rows_lo, int rows_hi,
                                             size_t S, int col, uint32_t bm) {
  for (int a = rows_lo; a < rows_hi; a++) {
    uint32_t* p = reinterpret_cast<uint32_t*>(base + (size_t)a * S) + col;
    uint32_t v = src[a] * 0x01010101u;
    *p = bm == 0xFFFFFFFFu ? v : ((*p & ~bm) | (v & bm));
  }
}

__global__ void restore_kernel(DevState st, Snapshot snap, const uint8_t* __restrict__ mask,
                               int mem_chunks, int ram_chunks) {
  const size_t S = (size_t)st.S;
  const int col = blockIdx.x * blockDim.x + threadIdx.x;  // 4-env column
  if (col * 4 >= st.n) return;
  const uint32_t bm = mask4(mask, st.n, col * 4);
  if (bm == 0) return;
  const int chunk = blockIdx.y;
  if (chunk < mem_chunks) {
    int lo = chunk * ROW_CHUNK;
    restore_rows(st.mem, snap.mem, lo, lo + ROW_CHUNK, S, col, bm);
    return;
  }
  int c = chunk - mem_chunks;
  if (c < ram_chunks) {
    int lo = c * ROW_CHUNK, hi = lo + ROW_CHUNK < snap.ram_bytes ? lo + ROW_CHUNK : snap.ram_bytes;
    restore_rows(st.cart_ram, snap.cart_ram, lo, hi, S, col, bm);
    return;
  }
  c -= ram_chunks;
  if (c < SERIAL_MAX / ROW_CHUNK) {
    restore_rows(st.serial, snap.serial, c * ROW_CHUNK, (c + 1) * ROW_CHUNK, S, col, bm);
    return;
  }
  // scalars: one thread handles its four envs
  for (int k = 0; k < 4; k++) {
    const int e = col * 4 + k;
    if (!((bm >> (8 * k)) & 0xFF)) continue;
    for (int f = 0; f < CS_STRIDE; f++) st.cart_state[(size_t)f * S + e] = snap.cart_state[f];
    for (int f = 0; f < I32_COUNT; f++) st.i32[(size_t)f * S + e] = snap.i32[f];
    for (int f = 0; f < I64_COUNT; f++) st.i64[(size_t)f * S + e] = snap.i64[f];
    for (int f = 0; f < U8_COUNT; f++) st.u8s[(size_t)f * S + e] = snap.u8s[f];
  }
}

// --- layout conversion for host export -------------------------------------------
// dst[(e - lo) * rows + a] = src[a * S + e] for e in [lo, hi), a in [0, rows)
__global__ void to_env_major_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int rows,
                                    size_t S, int lo, int hi) {
  __shared__ uint8_t tile[32][33];
  const int a0 = blockIdx.x * 32, e0 = lo + blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int k = ty; k < 32; k += 8) {
    int a = a0 + k, e = e0 + tx;
    tile[k][tx] = (a < rows && e < hi) ? src[(size_t)a * S + e] : 0;
  }
  __syncthreads();
  for (int k = ty; k < 32; k += 8) {
    int e = e0 + k, a = a0 + tx;
    if (a < rows && e < hi) dst[(size_t)(e - lo) * rows + a] = tile[tx][k];
  }
}

// src[(e - lo) * rows + a] -> dst[a * S + e]
__global__ void from_env_major_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int rows,
                                      size_t S, int lo, int hi) {
  __shared__ uint8_t tile[32][33];
  const int a0 = blockIdx.x * 32, e0 = lo + blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
  for (int k = ty; k < 32; k += 8) {
    int e = e0 + k, a = a0 + tx;
    tile[k][tx] = (a < rows && e < hi) ? src[(size_t)(e - lo) * rows + a] : 0;
  }
  __syncthreads();
  for (int k = ty; k < 32; k += 8) {
    int a = a0 + k, e = e0 + tx;
    if (a < rows && e < hi) dst[(size_t)a * S + e] = tile[tx][k];
  }
}

// --- launchers ---------------------------------------------------------------------
cudaError_t launch_init(const DevState& st, cudaStream_t s) {
  init_kernel<<<148 * 4, 256, 0, s>>>(st);
  return cudaGetLastError();
}

cudaError_t launch_snapshot(const DevState& st, const Snapshot& snap, int env, cudaStream_t s) {
  snapshot_kernel<<<64, 256, 0, s>>>(st, snap, env);
  return cudaGetLastError();
}

cudaError_t launch_restore(const DevState& st, const Snapshot& snap, const uint8_t* mask, cudaStream_t s) {
  const int cols = (st.n + 3) / 4;
  const int mem_chunks = MEM_SIZE / ROW_CHUNK;
  const int ram_chunks = (snap.ram_bytes + ROW_CHUNK - 1) / ROW_CHUNK;
  dim3 grid((cols + 127) / 128, mem_chunks + ram_chunks + SERIAL_MAX / ROW_CHUNK + 1);
  restore_kernel<<<grid, 128, 0, s>>>(st, snap, mask, mem_chunks, ram_chunks);
  return cudaGetLastError();
}

cudaError_t launch_to_env_major(const uint8_t* src, uint8_t* dst, int rows, int S, int lo, int hi,
                                cudaStream_t s) {
  dim3 grid((rows + 31) / 32, (hi - lo + 31) / 32);
  to_env_major_kernel<<<grid, dim3(32, 8), 0, s>>>(src, dst, rows, (size_t)S, lo, hi);
  return cudaGetLastError();
}

cudaError_t launch_from_env_major(const uint8_t* src, uint8_t* dst, int rows, int S, int lo, int hi,
                                  cudaStream_t s) {
  dim3 grid((rows + 31) / 32, (hi - lo + 31) / 32);
  from_env_major_kernel<<<grid, dim3(32, 8), 0, s>>>(src, dst, rows, (size_t)S, lo, hi);
  return cudaGetLastError();
}

}  // namespace gbx
