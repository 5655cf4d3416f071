// gbx_state.cu - whole-state kernels: initial state, snapshot capture and the
// masked restore.
//
// The masked restore replaces the reference's ~37 launches of
// reset_copy_{strided,scalar}_* (src/gbxcule/kernels/reset_mask.py:12-79,
// driven by src/gbxcule/core/reset_cache.py:192-307) with one launch. It
// restores exactly the fields ResetCache restores: the 64 KiB address space,
// cart_state, cart RAM, the serial buffer, the 72x80 shade image when the
// batch has one (reset_cache.py:111-112,237-244) and every per-env scalar,
// including the host-path action buffer; env-0 latches, obs, reward and the
// packed image are untouched.
//
// With env-major byte arrays a restored env is three contiguous blocks
// (64 KiB + cart RAM + 1 KiB), so the restore is a streaming copy: a grid of
// persistent blocks shares out the envs, each block reads the mask bytes of
// up to 256 of its envs at once, lists the masked ones, and copies each with
// the whole block, four 16-byte loads in flight per thread. The snapshot
// source stays resident in L2, so HBM sees the writes only (plus one read of
// the snapshot).
#include <cuda_runtime.h>
#include <stdint.h>

#include "gbx_layout.h"

namespace gbx {

constexpr int RESTORE_THREADS = 256;

// --- initial state (src/gbxcule/backends/warp_vec.py:249-497) ---------------
// Expects every buffer zeroed beforehand: the boot ROM goes to 0x0000-0x00FF
// of every env, and the cart_state / joypad-select defaults are set.
__global__ void init_kernel(DevState st) {
  const size_t S = (size_t)st.S;
  const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const uint4* boot4 = reinterpret_cast<const uint4*>(st.boot);
  for (long long k = tid; k < (long long)st.n * 16; k += stride) {
    const long long e = k >> 4;
    const int part = (int)(k & 15);
    reinterpret_cast<uint4*>(st.mem + (size_t)e * MEM_SIZE)[part] = boot4[part];
  }
  for (long long e = tid; e < st.n; e += stride) {
    st.cart_state[(size_t)CS_MBC_KIND * S + e] = st.mbc_kind;
    st.cart_state[(size_t)CS_ROM_BANK_LO * S + e] = 1;
    st.cart_state[(size_t)CS_BOOTROM * S + e] = 1;
    st.u8s[(size_t)F_JOYP_SELECT * S + e] = 0x30;
  }
}

// Block-wide copy of `bytes` bytes; 16-byte vectors when both ends and the
// length allow it (every block of the env-major arrays is 16-byte aligned
// except cart RAM of a cartridge without RAM, one byte per env).
__device__ __forceinline__ void block_copy(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src,
                                           int bytes) {
  if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | (uintptr_t)bytes) & 15) == 0) {
    uint4* __restrict__ d = reinterpret_cast<uint4*>(dst);
    const uint4* __restrict__ s = reinterpret_cast<const uint4*>(src);
    const int n16 = bytes / 16, step = blockDim.x;
    int k = threadIdx.x;
    for (; k + 3 * step < n16; k += 4 * step) {  // four loads in flight before the stores
      const uint4 a = s[k], b = s[k + step], c = s[k + 2 * step], e = s[k + 3 * step];
      d[k] = a; d[k + step] = b; d[k + 2 * step] = c; d[k + 3 * step] = e;
    }
    for (; k < n16; k += step) d[k] = s[k];
  } else {
    for (int k = threadIdx.x; k < bytes; k += blockDim.x) dst[k] = src[k];
  }
}

// --- snapshot capture (reset_cache.py:67-190) ----------------------------------
__global__ void snapshot_kernel(DevState st, Snapshot snap, int env) {
  const size_t S = (size_t)st.S;
  block_copy(snap.mem, st.mem + (size_t)env * MEM_SIZE, MEM_SIZE);
  block_copy(snap.cart_ram, st.cart_ram + (size_t)env * st.ram_rows, snap.ram_bytes);
  block_copy(snap.serial, st.serial + (size_t)env * SERIAL_MAX, SERIAL_MAX);
  if (snap.pix && st.pix) block_copy(snap.pix, st.pix + (size_t)env * SHADE_BYTES, SHADE_BYTES);
  const int t = threadIdx.x;
  if (t < CS_STRIDE) snap.cart_state[t] = st.cart_state[(size_t)t * S + env];
  if (t < I32_COUNT) snap.i32[t] = st.i32[(size_t)t * S + env];
  if (t < I64_COUNT) snap.i64[t] = st.i64[(size_t)t * S + env];
  if (t < U8_COUNT) snap.u8s[t] = st.u8s[(size_t)t * S + env];
}

// --- masked restore ------------------------------------------------------------
__global__ void __launch_bounds__(RESTORE_THREADS) restore_kernel(DevState st, Snapshot snap,
                                                                  const uint8_t* __restrict__ mask) {
  const size_t S = (size_t)st.S;
  // this block's envs are blockIdx.x + j * gridDim.x; read their mask bytes
  // at once and list the masked ones
  __shared__ int list[RESTORE_THREADS];
  __shared__ int count;
  for (int j0 = 0; blockIdx.x + j0 * gridDim.x < st.n; j0 += RESTORE_THREADS) {
    if (threadIdx.x == 0) count = 0;
    __syncthreads();
    const int e_t = blockIdx.x + (j0 + threadIdx.x) * gridDim.x;
    if (e_t < st.n && mask[e_t]) list[atomicAdd(&count, 1)] = e_t;
    __syncthreads();
    const int cnt = count;
    for (int q = 0; q < cnt; q++) {
      const int e = list[q];
      block_copy(st.mem + (size_t)e * MEM_SIZE, snap.mem, MEM_SIZE);
      block_copy(st.cart_ram + (size_t)e * st.ram_rows, snap.cart_ram, snap.ram_bytes);
      block_copy(st.serial + (size_t)e * SERIAL_MAX, snap.serial, SERIAL_MAX);
      if (snap.pix && st.pix) block_copy(st.pix + (size_t)e * SHADE_BYTES, snap.pix, SHADE_BYTES);
      const int t = threadIdx.x;
      if (t < CS_STRIDE) st.cart_state[(size_t)t * S + e] = snap.cart_state[t];
      if (t < I32_COUNT) st.i32[(size_t)t * S + e] = snap.i32[t];
      if (t < I64_COUNT) st.i64[(size_t)t * S + e] = snap.i64[t];
      if (t < U8_COUNT) st.u8s[(size_t)t * S + e] = snap.u8s[t];
    }
    __syncthreads();  // list and count are reused by the next batch
  }
}

// --- launchers ---------------------------------------------------------------------
cudaError_t launch_init(const DevState& st, cudaStream_t s, int sms) {
  init_kernel<<<(sms > 0 ? sms : 1) * 4, 256, 0, s>>>(st);
  return cudaGetLastError();
}

cudaError_t launch_snapshot(const DevState& st, const Snapshot& snap, int env, cudaStream_t s) {
  snapshot_kernel<<<1, 1024, 0, s>>>(st, snap, env);
  return cudaGetLastError();
}

cudaError_t launch_restore(const DevState& st, const Snapshot& snap, const uint8_t* mask, cudaStream_t s,
                           int sms) {
  // 8 resident 256-thread blocks per SM; fewer blocks than envs keeps the
  // mask scan cheap when few envs are masked
  const int slots = (sms > 0 ? sms : 1) * 8;
  const int blocks = st.n < slots ? st.n : slots;
  restore_kernel<<<blocks, RESTORE_THREADS, 0, s>>>(st, snap, mask);
  return cudaGetLastError();
}

}  // namespace gbx
