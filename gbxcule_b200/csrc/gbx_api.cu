// gbx_api.cu - the C ABI (include/gbx.h): handle lifetime, device buffers,
// launches and host transfers. No exception crosses the boundary; every entry
// point returns a gbx_status and leaves a message in gbx_last_error().
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <new>
#include <string>

#include "../../include/gbx.h"
#include "gbx_layout.h"

namespace gbx {
cudaError_t launch_step(const DevState& st, const uint32_t* pre, const int32_t* actions, int frames, int release,
                        int stage, cudaStream_t stream, const DebugCfg& dbg, int K, int sms, bool uniform);
int fill_envs_per_warp(long long n, int sms);
int envs_per_warp_override();
int dispatch_override();
cudaError_t launch_render_bg_env0(const DevState& st, uint8_t* out, cudaStream_t stream);
void predecode_rom(const uint8_t* rom, int n, uint32_t* out);
cudaError_t launch_render(const DevState& st, uint8_t* out, int64_t base_offset, bool packed,
                          cudaStream_t stream, uint16_t* scaled, uint64_t scale_tab, int s2d);
cudaError_t launch_init(const DevState& st, cudaStream_t s, int sms);
cudaError_t launch_snapshot(const DevState& st, const Snapshot& snap, int env, cudaStream_t s);
cudaError_t launch_restore(const DevState& st, const Snapshot& snap, const uint8_t* mask, cudaStream_t s,
                           int sms);
}  // namespace gbx

using namespace gbx;

static_assert((int)GBX_I32_COUNT == (int)I32_COUNT, "i32 field table mismatch");
static_assert((int)GBX_I64_COUNT == (int)I64_COUNT, "i64 field table mismatch");
static_assert((int)GBX_U8_COUNT == (int)U8_COUNT, "u8 field table mismatch");

// Launch shape of the step kernel, chosen per handle: envs per warp K and
// the interpreter (switch or uniform datapath). Neither changes a result.
// A shape is coded as K | UNI_BIT. Automatic mode times its candidates on the
// handle's first real steps, in the order A B B A (A B C C B A, ...) so that
// a step time drifting as the envs diverge weighs on every candidate alike,
// and keeps the fastest. Timing uses events around the step launches already
// requested; no step is added or repeated.
constexpr int UNI_BIT = 64;
inline int shape_k(int m) { return m & 63; }
inline bool shape_uni(int m) { return (m & UNI_BIT) != 0; }
struct KTuner {
  static constexpr int MAXC = 5;
  int fixed = 0;              // > 0: K set by the caller or GBX_ENVS_PER_WARP
  int disp = 0;               // gbx_dispatch set by the caller or GBX_DISPATCH
  int ncand = 0, cand[MAXC] = {};
  int order[2 * MAXC] = {};
  int launched = 0;           // trials launched (events recorded)
  int measured = 0;           // trials whose events were read
  float ms[MAXC] = {};
  cudaEvent_t ev[2 * MAXC][2] = {};
  int best = 0;               // chosen shape once every trial is measured
  bool settled() const { return ncand <= 1 || measured == 2 * ncand; }
};

struct gbx_env {
  DevState st;
  gbx_config cfg;
  int32_t ram_bytes;       // cartridge RAM bytes per env (0 if none)
  int32_t ram_rows;        // max(ram_bytes, 1): rows allocated/snapshotted
  uint8_t* pix;
  uint8_t* pix_packed;
  uint32_t* pre;           // pre-decoded ROM, one word per byte (gbx_step.cu)
  uint8_t* frame_bg;       // env-0 160x144 frame
  DebugCfg dbg;            // debug traps (all off by default)
  bool initialized;
  int sm_count;            // SMs of the handle's device
  KTuner tune;
  int last_shape;          // launch shape of the latest step launch (0: none yet)
  // Owners: the creator (dropped by gbx_destroy) plus one per live DLPack
  // tensor (dropped by its deleter). Device memory is freed with the last.
  std::atomic<int> refs;
};

struct gbx_snapshot {
  Snapshot s;
  void* block;
  int device;
};

namespace {

thread_local std::string g_err;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_err = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(e == cudaErrorMemoryAllocation ? GBX_ERR_OOM : GBX_ERR_CUDA, "%s: %s", what,
              cudaGetErrorString(e));
}

#define CK(call, what)                          \
  do {                                          \
    cudaError_t e_ = (call);                    \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

inline cudaStream_t S_(void* s) { return reinterpret_cast<cudaStream_t>(s); }

const int kRomSizes[][2] = {{0x00, 32 << 10}, {0x01, 64 << 10}, {0x02, 128 << 10}, {0x03, 256 << 10},
                            {0x04, 512 << 10}, {0x05, 1 << 20}, {0x06, 2 << 20}, {0x07, 4 << 20},
                            {0x08, 8 << 20}, {0x52, 1153433}, {0x53, 1258291}, {0x54, 1572864}};
const int kRamSizes[][2] = {{0x00, 0}, {0x01, 2 << 10}, {0x02, 8 << 10}, {0x03, 32 << 10},
                            {0x04, 128 << 10}, {0x05, 64 << 10}};

// src/gbxcule/core/cartridge.py:139-187
int parse_header(const uint8_t* rom, size_t len, int* mbc, int* rom_bytes, int* ram_bytes) {
  if (len < 0x150) return fail(GBX_ERR_INVALID, "ROM too small for header: %zu bytes", len);
  int ct = rom[0x147];
  if (ct == 0x00) *mbc = MBC_ROM_ONLY;
  else if (ct >= 0x01 && ct <= 0x03) *mbc = MBC_MBC1;
  else if (ct >= 0x0F && ct <= 0x13) *mbc = MBC_MBC3;
  else return fail(GBX_ERR_INVALID, "Unsupported cartridge type: 0x%02X", ct);
  *rom_bytes = -1;
  for (auto& r : kRomSizes) if (r[0] == rom[0x148]) *rom_bytes = r[1];
  if (*rom_bytes < 0) return fail(GBX_ERR_INVALID, "Unsupported ROM size code: 0x%02X", rom[0x148]);
  if (*rom_bytes % ROM_BANK) return fail(GBX_ERR_INVALID, "Invalid ROM byte length: %d", *rom_bytes);
  *ram_bytes = -1;
  for (auto& r : kRamSizes) if (r[0] == rom[0x149]) *ram_bytes = r[1];
  if (*ram_bytes < 0) return fail(GBX_ERR_INVALID, "Unsupported RAM size code: 0x%02X", rom[0x149]);
  if (*ram_bytes % RAM_BANK) return fail(GBX_ERR_INVALID, "Invalid RAM byte length: %d", *ram_bytes);
  if (len < (size_t)*rom_bytes)
    return fail(GBX_ERR_INVALID, "ROM smaller than header advertises: %zu < %d", len, *rom_bytes);
  return GBX_OK;
}

template <class T>
int dalloc(T** p, size_t count) {
  *p = nullptr;
  if (count == 0) count = 1;
  cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMalloc");
  return GBX_OK;
}

void free_env(gbx_env* h) {
  DevState& st = h->st;
  void* ptrs[] = {(void*)st.rom, (void*)st.boot, st.mem, st.cart_ram, st.serial, st.cart_state, st.i32,
                  st.i64, st.u8s, st.latch, st.obs, st.reward, st.status, h->pix, h->pix_packed, h->pre,
                  h->frame_bg};
  for (void* p : ptrs)
    if (p) cudaFree(p);
  for (auto& pair : h->tune.ev)
    for (cudaEvent_t& e : pair)
      if (e) cudaEventDestroy(e);
}

// Candidates of the automatic choice for n envs on `sms` SMs. K: the one
// that fills one wave of warps, half of it (two waves of emptier warps) and
// 32, or the fixed K. Interpreter: the switch at every candidate K, the
// uniform datapath at the K that fill warps at least half (with fewer lanes
// a fixed datapath wastes most of its issue slots), or the fixed one.
void tuner_init(KTuner& t, int n, int sms, int fixed, int disp) {
  t = KTuner();
  t.fixed = fixed;
  t.disp = disp;
  int ks[3] = {0, 0, 0}, nk = 0;
  const int kf = fill_envs_per_warp(n, sms);
  if (fixed) ks[nk++] = fixed;
  else {
    ks[nk++] = kf;
    if (kf > 1) ks[nk++] = kf / 2;
    if (kf < 32) ks[nk++] = 32;
  }
  for (int i = 0; i < nk; i++)
    if (disp != GBX_DISPATCH_UNIFORM && t.ncand < KTuner::MAXC) t.cand[t.ncand++] = ks[i];
  for (int i = 0; i < nk; i++)
    if ((disp == GBX_DISPATCH_UNIFORM || (disp == GBX_DISPATCH_AUTO && ks[i] >= 16)) && t.ncand < KTuner::MAXC)
      t.cand[t.ncand++] = ks[i] | UNI_BIT;
  for (int i = 0; i < t.ncand; i++) {
    t.order[i] = i;
    t.order[2 * t.ncand - 1 - i] = i;
  }
  t.best = t.cand[0];
}

// Read the events of finished trials; once all are read, keep the fastest K.
void tuner_poll(KTuner& t) {
  while (t.measured < t.launched) {
    cudaEvent_t* e = t.ev[t.measured];
    if (cudaEventQuery(e[1]) != cudaSuccess) { cudaGetLastError(); return; }  // not finished yet
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, e[0], e[1]) != cudaSuccess) { cudaGetLastError(); ms = 1e30f; }
    t.ms[t.order[t.measured]] += ms;
    t.measured++;
  }
  if (t.ncand > 1 && t.measured == 2 * t.ncand) {
    int b = 0;
    for (int i = 1; i < t.ncand; i++)
      if (t.ms[i] < t.ms[b]) b = i;
    t.best = t.cand[b];
  }
}

int zero_state(gbx_env* h, cudaStream_t s) {
  DevState& st = h->st;
  const size_t S = st.S, n = st.n;
  CK(cudaMemsetAsync(st.mem, 0, (size_t)MEM_SIZE * n, s), "memset mem");
  CK(cudaMemsetAsync(st.cart_ram, 0, (size_t)h->ram_rows * n, s), "memset cart_ram");
  CK(cudaMemsetAsync(st.serial, 0, (size_t)SERIAL_MAX * n, s), "memset serial");
  CK(cudaMemsetAsync(st.cart_state, 0, sizeof(int32_t) * CS_STRIDE * S, s), "memset cart_state");
  CK(cudaMemsetAsync(st.i32, 0, sizeof(int32_t) * I32_COUNT * S, s), "memset i32");
  CK(cudaMemsetAsync(st.i64, 0, sizeof(int64_t) * I64_COUNT * S, s), "memset i64");
  CK(cudaMemsetAsync(st.u8s, 0, (size_t)U8_COUNT * S, s), "memset u8");
  CK(cudaMemsetAsync(st.latch, 0, 9 * SCREEN_H, s), "memset latch");
  CK(cudaMemsetAsync(h->frame_bg, 0, 160 * SCREEN_H, s), "memset frame_bg");
  CK(cudaMemsetAsync(st.obs, 0, sizeof(float) * OBS_DIM * (size_t)st.n, s), "memset obs");
  CK(cudaMemsetAsync(st.reward, 0, sizeof(float) * (size_t)st.n, s), "memset reward");
  CK(cudaMemsetAsync(st.status, 0, sizeof(uint32_t), s), "memset status");
  if (h->pix) CK(cudaMemsetAsync(h->pix, 0, (size_t)SHADE_BYTES * st.n, s), "memset pix");
  if (h->pix_packed) CK(cudaMemsetAsync(h->pix_packed, 0, (size_t)PACKED_BYTES * st.n, s), "memset pix_packed");
  return GBX_OK;
}

// Drop one owner; the last one frees every device buffer. cudaFree waits for
// the device's outstanding work, as the callers' declarations state.
void env_release(gbx_env* h) {
  if (h->refs.fetch_sub(1, std::memory_order_acq_rel) != 1) return;
  DeviceGuard g(h->cfg.device);
  cudaDeviceSynchronize();
  free_env(h);
  delete h;
}

int check_env(const gbx_env* h) {
  if (!h) return fail(GBX_ERR_INVALID, "null gbx_env");
  return GBX_OK;
}
int check_init(const gbx_env* h) {
  if (!h) return fail(GBX_ERR_INVALID, "null gbx_env");
  if (!h->initialized) return fail(GBX_ERR_STATE, "Backend not initialized. Call reset() first.");
  return GBX_OK;
}
int check_range(const gbx_env* h, int lo, int hi) {
  if (lo < 0 || hi > h->st.n || lo > hi)
    return fail(GBX_ERR_RANGE, "env range [%d, %d) out of range [0, %d)", lo, hi, h->st.n);
  return GBX_OK;
}

// env-major byte arrays [n][rows]: envs [lo, hi) are one contiguous range
int export_rows(const uint8_t* src, int rows, int lo, int hi, uint8_t* host) {
  if (hi > lo)
    CK(cudaMemcpy(host, src + (size_t)lo * rows, (size_t)(hi - lo) * rows, cudaMemcpyDeviceToHost), "export copy");
  return GBX_OK;
}
int import_rows(uint8_t* dst, int rows, int lo, int hi, const uint8_t* host) {
  if (hi > lo)
    CK(cudaMemcpy(dst + (size_t)lo * rows, host, (size_t)(hi - lo) * rows, cudaMemcpyHostToDevice), "import copy");
  return GBX_OK;
}
template <class T>
int copy_fields(T* dev, int fields, size_t S, int lo, int hi, T* host, bool to_host) {
  size_t w = sizeof(T) * (size_t)(hi - lo);
  if (w == 0) return GBX_OK;
  if (to_host)
    CK(cudaMemcpy2D(host, w, dev + lo, sizeof(T) * S, w, fields, cudaMemcpyDeviceToHost), "field copy");
  else
    CK(cudaMemcpy2D(dev + lo, sizeof(T) * S, host, w, w, fields, cudaMemcpyHostToDevice), "field copy");
  return GBX_OK;
}

}  // namespace

#define RET(x)                     \
  do {                             \
    int r_ = (x);                  \
    if (r_ != GBX_OK) return r_;   \
  } while (0)

extern "C" {

int32_t gbx_abi_version(void) { return GBX_ABI_VERSION; }

const char* gbx_last_error(void) { return g_err.c_str(); }

int gbx_create(const gbx_config* cfg, const uint8_t* rom, size_t rom_len, const uint8_t* boot, size_t boot_len,
               gbx_env** out) {
  if (!cfg || !rom || !boot || !out) return fail(GBX_ERR_INVALID, "null argument to gbx_create");
  *out = nullptr;
  if (cfg->num_envs <= 0) return fail(GBX_ERR_INVALID, "num_envs must be > 0, got %d", cfg->num_envs);
  if (cfg->stage < 0 || cfg->stage > 3) return fail(GBX_ERR_INVALID, "unknown stage %d", cfg->stage);
  if (boot_len != 0x100) return fail(GBX_ERR_INVALID, "Boot ROM must be 256 bytes, got %zu", boot_len);
  int mbc, rom_bytes, ram_bytes;
  RET(parse_header(rom, rom_len, &mbc, &rom_bytes, &ram_bytes));
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || cfg->device < 0 || cfg->device >= ndev)
    return fail(GBX_ERR_INVALID, "CUDA device %d not available (%d devices)", cfg->device, ndev);
  DeviceGuard g(cfg->device);
  gbx_env* h = new (std::nothrow) gbx_env();
  if (!h) return fail(GBX_ERR_OOM, "host allocation failed");
  h->refs.store(1);
  h->cfg = *cfg;
  DevState& st = h->st;
  st.n = cfg->num_envs;
  st.S = (cfg->num_envs + 127) & ~127;
  st.mbc_kind = mbc;
  st.rom_bytes = rom_bytes;
  st.rom_bank_count = rom_bytes / ROM_BANK;
  st.rom_bank_mask = (st.rom_bank_count & (st.rom_bank_count - 1)) == 0 ? st.rom_bank_count - 1 : -1;
  st.ram_bank_count = ram_bytes / RAM_BANK;
  h->ram_bytes = ram_bytes;
  h->ram_rows = ram_bytes > 0 ? ram_bytes : 1;
  st.ram_rows = h->ram_rows;
  const size_t S = st.S, n = st.n;
  int rc = GBX_OK;
  uint8_t *rom_d = nullptr, *boot_d = nullptr;
  // the ROM is padded with 16 zero bytes: the uniform interpreter fetches an
  // instruction as the two aligned words around it
  if ((rc = dalloc(&rom_d, (size_t)rom_bytes + 16)) || (rc = dalloc(&boot_d, 256)) ||
      (rc = dalloc(&st.mem, (size_t)MEM_SIZE * n)) || (rc = dalloc(&st.cart_ram, (size_t)h->ram_rows * n)) ||
      (rc = dalloc(&st.serial, (size_t)SERIAL_MAX * n)) || (rc = dalloc(&st.cart_state, (size_t)CS_STRIDE * S)) ||
      (rc = dalloc(&st.i32, (size_t)I32_COUNT * S)) || (rc = dalloc(&st.i64, (size_t)I64_COUNT * S)) ||
      (rc = dalloc(&st.u8s, (size_t)U8_COUNT * S)) || (rc = dalloc(&st.latch, 9 * SCREEN_H)) ||
      (rc = dalloc(&st.obs, (size_t)OBS_DIM * st.n)) || (rc = dalloc(&st.reward, (size_t)st.n)) ||
      (rc = dalloc(&st.status, 1)) ||
      (cfg->alloc_pixels && (rc = dalloc(&h->pix, (size_t)SHADE_BYTES * st.n))) ||
      (cfg->alloc_pixels_packed && (rc = dalloc(&h->pix_packed, (size_t)PACKED_BYTES * st.n)))) {
    st.rom = rom_d;
    st.boot = boot_d;
    free_env(h);
    delete h;
    return rc;
  }
  st.rom = rom_d;
  st.boot = boot_d;
  st.pix = h->pix;
  if ((rc = dalloc(&h->frame_bg, (size_t)160 * SCREEN_H)) || (rc = dalloc(&h->pre, (size_t)rom_bytes))) {
    free_env(h);
    delete h;
    return rc;
  }
  uint32_t* pre_host = new (std::nothrow) uint32_t[rom_bytes];
  if (!pre_host) {
    free_env(h);
    delete h;
    return fail(GBX_ERR_OOM, "host allocation failed");
  }
  predecode_rom(rom, rom_bytes, pre_host);
  cudaError_t e = cudaMemcpy(rom_d, rom, (size_t)rom_bytes, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemset(rom_d + rom_bytes, 0, 16);
  if (e == cudaSuccess) e = cudaMemcpy(boot_d, boot, 256, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(h->pre, pre_host, sizeof(uint32_t) * rom_bytes, cudaMemcpyHostToDevice);
  delete[] pre_host;
  if (e != cudaSuccess) {
    free_env(h);
    delete h;
    return cuda_fail(e, "upload ROM");
  }
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, cfg->device) != cudaSuccess || sms <= 0) {
    free_env(h);
    delete h;
    return fail(GBX_ERR_CUDA, "cannot read the SM count of device %d", cfg->device);
  }
  h->sm_count = sms;
  tuner_init(h->tune, st.n, sms, envs_per_warp_override(), dispatch_override());
  *out = h;
  return GBX_OK;
}

int gbx_destroy(gbx_env* h) {
  if (!h) return GBX_OK;
  env_release(h);
  return GBX_OK;
}

int gbx_get_info(const gbx_env* h, gbx_info* out) {
  RET(check_env(h));
  if (!out) return fail(GBX_ERR_INVALID, "null out");
  out->num_envs = h->st.n;
  out->env_stride = h->st.S;
  out->device = h->cfg.device;
  out->stage = h->cfg.stage;
  out->mbc_kind = h->st.mbc_kind;
  out->rom_bytes = h->st.rom_bytes;
  out->rom_bank_count = h->st.rom_bank_count;
  out->rom_bank_mask = h->st.rom_bank_mask;
  out->ram_bank_count = h->st.ram_bank_count;
  out->ram_bytes = h->ram_bytes;
  out->sm_count = h->sm_count;
  tuner_poll(const_cast<gbx_env*>(h)->tune);  // trials that have finished since
  const int shape = h->last_shape ? h->last_shape : h->tune.best;
  out->envs_per_warp = shape_k(shape);
  out->envs_per_warp_tuned = h->tune.settled();
  out->dispatch = shape_uni(shape) ? GBX_DISPATCH_UNIFORM : GBX_DISPATCH_SWITCH;
  return GBX_OK;
}

int gbx_reset(gbx_env* h, void* stream) {
  RET(check_env(h));
  DeviceGuard g(h->cfg.device);
  cudaStream_t s = S_(stream);
  RET(zero_state(h, s));
  CK(launch_init(h->st, s, h->sm_count), "init kernel");
  h->initialized = true;
  if (h->cfg.stage == STAGE_OBS || h->cfg.stage == STAGE_FULL) {
    const int32_t* zero_actions = h->st.i32 + (size_t)F_ACTIONS * h->st.S;
    const int shape = h->tune.best;
    CK(launch_step(h->st, h->pre, zero_actions, 0, 0, h->cfg.stage, s, h->dbg, shape_k(shape), h->sm_count,
                   shape_uni(shape)),
       "step kernel (reset obs)");
  }
  return GBX_OK;
}

int gbx_step(gbx_env* h, const int32_t* actions, int32_t frames, int32_t release, void* stream) {
  RET(check_init(h));
  if (!actions) return fail(GBX_ERR_INVALID, "actions is null");
  if (frames < 0) return fail(GBX_ERR_INVALID, "frames_to_run must be >= 0, got %d", frames);
  if (frames > 25000) return fail(GBX_ERR_INVALID, "frames_to_run %d exceeds 25000 per launch", frames);
  DeviceGuard g(h->cfg.device);
  cudaStream_t s = S_(stream);
  KTuner& t = h->tune;
  cudaEvent_t* trial = nullptr;
  tuner_poll(t);
  int shape = t.best;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  // trials only on real steps, outside stream capture and debug traps
  if (t.ncand > 1 && t.launched < 2 * t.ncand && frames > 0 && !h->dbg.active() &&
      cudaStreamIsCapturing(s, &cap) == cudaSuccess && cap == cudaStreamCaptureStatusNone) {
    trial = t.ev[t.launched];
    for (int k = 0; k < 2; k++)
      if (!trial[k]) CK(cudaEventCreate(&trial[k]), "tuner event");
    shape = t.cand[t.order[t.launched]];
    CK(cudaEventRecord(trial[0], s), "tuner event record");
  }
  h->last_shape = shape;
  CK(launch_step(h->st, h->pre, actions, frames, release, h->cfg.stage, s, h->dbg, shape_k(shape),
                 h->sm_count, shape_uni(shape)),
     "step kernel");
  if (trial) {
    CK(cudaEventRecord(trial[1], s), "tuner event record");
    t.launched++;
  }
  return GBX_OK;
}

// New tuner state for a fixed K (0 = automatic) and dispatch (0 = automatic).
static void retune(gbx_env* h, int k, int disp) {
  DeviceGuard g(h->cfg.device);
  cudaDeviceSynchronize();  // no trial of the previous setting is still in flight
  KTuner fresh;
  tuner_init(fresh, h->st.n, h->sm_count, k, disp);
  for (int i = 0; i < 2 * KTuner::MAXC; i++)  // keep the created events
    for (int j = 0; j < 2; j++) fresh.ev[i][j] = h->tune.ev[i][j];
  h->tune = fresh;
  h->last_shape = 0;
}

int gbx_set_envs_per_warp(gbx_env* h, int32_t k) {
  RET(check_env(h));
  if (k < 0 || k > 32) return fail(GBX_ERR_INVALID, "envs_per_warp must be in [0, 32], got %d", k);
  retune(h, k, h->tune.disp);
  return GBX_OK;
}

int gbx_set_dispatch(gbx_env* h, int32_t d) {
  RET(check_env(h));
  if (d < GBX_DISPATCH_AUTO || d > GBX_DISPATCH_UNIFORM)
    return fail(GBX_ERR_INVALID, "dispatch must be 0 (auto), 1 (switch) or 2 (uniform), got %d", d);
  retune(h, h->tune.fixed, d);
  return GBX_OK;
}

int gbx_render_packed(gbx_env* h, uint8_t* out, int64_t base_offset, void* stream) {
  RET(check_init(h));
  if (base_offset < 0) return fail(GBX_ERR_INVALID, "base_offset_bytes must be >= 0");
  if (!out) {
    if (!h->pix_packed) return fail(GBX_ERR_STATE, "Packed pixel buffer not initialized. Call reset() first.");
    out = h->pix_packed;
    base_offset = 0;
  }
  DeviceGuard g(h->cfg.device);
  CK(launch_render(h->st, out, base_offset, true, S_(stream), nullptr, 0, 0), "render kernel");
  return GBX_OK;
}

// bf16 bits of (float)v, rounded to nearest even (v finite)
static uint16_t bf16_bits(float v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

int gbx_render_packed_scaled(gbx_env* h, uint8_t* out, int64_t base_offset, void* scaled, int32_t layout,
                             void* stream) {
  RET(check_init(h));
  if (base_offset < 0) return fail(GBX_ERR_INVALID, "base_offset_bytes must be >= 0");
  if (layout != 0 && layout != 1) return fail(GBX_ERR_INVALID, "layout must be 0 (rows) or 1 (space-to-depth), got %d", layout);
  if (!scaled) return fail(GBX_ERR_INVALID, "scaled output is null");
  if (reinterpret_cast<uintptr_t>(scaled) & 15) return fail(GBX_ERR_INVALID, "scaled output must be 16-byte aligned");
  if (!out) {
    if (!h->pix_packed) return fail(GBX_ERR_STATE, "Packed pixel buffer not initialized. Call reset() first.");
    out = h->pix_packed;
    base_offset = 0;
  }
  uint64_t tab = 0;
  for (int v = 0; v < 4; v++) tab |= (uint64_t)bf16_bits((float)v / 3.0f) << (16 * v);
  DeviceGuard g(h->cfg.device);
  CK(launch_render(h->st, out, base_offset, true, S_(stream), static_cast<uint16_t*>(scaled), tab, layout),
     "render kernel");
  return GBX_OK;
}

int gbx_render_shades(gbx_env* h, uint8_t* out, void* stream) {
  RET(check_init(h));
  if (!out) {
    if (!h->pix) return fail(GBX_ERR_STATE, "Pixel buffer not initialized. Call reset() first.");
    out = h->pix;
  }
  DeviceGuard g(h->cfg.device);
  CK(launch_render(h->st, out, 0, false, S_(stream), nullptr, 0, 0), "render kernel");
  return GBX_OK;
}

int gbx_snapshot_create(gbx_env* h, int32_t env_idx, void* stream, gbx_snapshot** out) {
  RET(check_init(h));
  if (!out) return fail(GBX_ERR_INVALID, "null out");
  *out = nullptr;
  if (env_idx < 0 || env_idx >= h->st.n)
    return fail(GBX_ERR_RANGE, "env_idx %d out of range [0, %d)", env_idx, h->st.n);
  DeviceGuard g(h->cfg.device);
  gbx_snapshot* sn = new (std::nothrow) gbx_snapshot();
  if (!sn) return fail(GBX_ERR_OOM, "host allocation failed");
  const size_t pix_bytes = h->pix ? (size_t)SHADE_BYTES : 0;
  const size_t bytes = (size_t)MEM_SIZE + h->ram_rows + SERIAL_MAX + pix_bytes + 4 * CS_STRIDE + 4 * I32_COUNT +
                       8 * I64_COUNT + U8_COUNT + 64;
  cudaError_t e = cudaMalloc(&sn->block, bytes);
  if (e != cudaSuccess) {
    delete sn;
    return cuda_fail(e, "snapshot alloc");
  }
  // byte blocks first so each starts 16-byte aligned (cart RAM sizes are
  // multiples of 16 or a single byte)
  uint8_t* p = static_cast<uint8_t*>(sn->block);
  sn->s.mem = p; p += MEM_SIZE;
  sn->s.serial = p; p += SERIAL_MAX;
  sn->s.pix = h->pix ? p : nullptr; p += pix_bytes;  // 5760: keeps 16-byte alignment
  sn->s.cart_ram = p; p += (h->ram_rows + 15) & ~15;
  sn->s.i64 = reinterpret_cast<int64_t*>(p); p += 8 * I64_COUNT;
  sn->s.cart_state = reinterpret_cast<int32_t*>(p); p += 4 * CS_STRIDE;
  sn->s.i32 = reinterpret_cast<int32_t*>(p); p += 4 * I32_COUNT;
  sn->s.u8s = p;
  sn->s.ram_bytes = h->ram_rows;
  sn->device = h->cfg.device;
  e = launch_snapshot(h->st, sn->s, env_idx, S_(stream));
  if (e != cudaSuccess) {
    cudaFree(sn->block);
    delete sn;
    return cuda_fail(e, "snapshot kernel");
  }
  *out = sn;
  return GBX_OK;
}

int gbx_snapshot_destroy(gbx_snapshot* sn) {
  if (!sn) return GBX_OK;
  DeviceGuard g(sn->device);
  cudaDeviceSynchronize();
  cudaFree(sn->block);
  delete sn;
  return GBX_OK;
}

int gbx_masked_restore(gbx_env* h, const gbx_snapshot* sn, const uint8_t* mask, void* stream) {
  RET(check_init(h));
  if (!sn || !mask) return fail(GBX_ERR_INVALID, "null snapshot or mask");
  if (sn->device != h->cfg.device || sn->s.ram_bytes != h->ram_rows)
    return fail(GBX_ERR_INVALID, "snapshot belongs to a different env batch");
  DeviceGuard g(h->cfg.device);
  CK(launch_restore(h->st, sn->s, mask, S_(stream), h->sm_count), "restore kernel");
  return GBX_OK;
}

int gbx_buffer(const gbx_env* h, int32_t which, gbx_buffer_info* o) {
  RET(check_env(h));
  if (!o) return fail(GBX_ERR_INVALID, "null out");
  memset(o, 0, sizeof *o);
  const DevState& st = h->st;
  const int64_t n = st.n, S = st.S;
  auto set = [&](void* d, int code, int bits, int nd, int64_t s0, int64_t s1, int64_t s2, int64_t t0, int64_t t1,
                 int64_t t2) {
    o->data = d; o->dtype_code = code; o->dtype_bits = bits; o->ndim = nd;
    o->shape[0] = s0; o->shape[1] = s1; o->shape[2] = s2;
    o->strides[0] = t0; o->strides[1] = t1; o->strides[2] = t2;
  };
  switch (which) {
    case GBX_BUF_MEM: set(st.mem, 1, 8, 2, n, MEM_SIZE, 0, MEM_SIZE, 1, 0); break;
    case GBX_BUF_PIXELS:
      if (!h->pix) return fail(GBX_ERR_STATE, "Pixel buffer not initialized. Call reset() first.");
      set(h->pix, 1, 8, 3, n, 72, 80, SHADE_BYTES, 80, 1); break;
    case GBX_BUF_PIXELS_PACKED:
      if (!h->pix_packed) return fail(GBX_ERR_STATE, "Packed pixel buffer not initialized. Call reset() first.");
      set(h->pix_packed, 1, 8, 3, n, 72, 20, PACKED_BYTES, 20, 1); break;
    case GBX_BUF_OBS: set(st.obs, 2, 32, 2, n, OBS_DIM, 0, OBS_DIM, 1, 0); break;
    case GBX_BUF_REWARD: set(st.reward, 2, 32, 1, n, 0, 0, 1, 0, 0); break;
    case GBX_BUF_CART_RAM: set(st.cart_ram, 1, 8, 2, n, h->ram_rows, 0, h->ram_rows, 1, 0); break;
    case GBX_BUF_SERIAL: set(st.serial, 1, 8, 2, n, SERIAL_MAX, 0, SERIAL_MAX, 1, 0); break;
    case GBX_BUF_I32: set(st.i32, 0, 32, 2, I32_COUNT, n, 0, S, 1, 0); break;
    case GBX_BUF_I64: set(st.i64, 0, 64, 2, I64_COUNT, n, 0, S, 1, 0); break;
    case GBX_BUF_U8: set(st.u8s, 1, 8, 2, U8_COUNT, n, 0, S, 1, 0); break;
    case GBX_BUF_CART_STATE: set(st.cart_state, 0, 32, 2, CS_STRIDE, n, 0, S, 1, 0); break;
    case GBX_BUF_LATCH: set(st.latch, 1, 8, 2, 9, SCREEN_H, 0, SCREEN_H, 1, 0); break;
    case GBX_BUF_FRAME_BG: set(h->frame_bg, 1, 8, 2, SCREEN_H, 160, 0, 160, 1, 0); break;
    default: return fail(GBX_ERR_INVALID, "unknown buffer id %d", which);
  }
  return GBX_OK;
}

// A DLPack tensor owns a reference to its handle (manager_ctx), so a view
// held past gbx_destroy keeps the device memory it aliases alive.
static void dl_deleter(DLManagedTensor* t) {
  gbx_env* h = static_cast<gbx_env*>(t->manager_ctx);
  free(t);
  if (h) env_release(h);
}

int gbx_export_dlpack(const gbx_env* h, int32_t which, void** out) {
  if (!out) return fail(GBX_ERR_INVALID, "null out");
  *out = nullptr;
  gbx_buffer_info b;
  RET(gbx_buffer(h, which, &b));
  // one block: tensor, then shape[3], strides[3]
  DLManagedTensor* t = static_cast<DLManagedTensor*>(malloc(sizeof(DLManagedTensor) + 6 * sizeof(int64_t)));
  if (!t) return fail(GBX_ERR_OOM, "host allocation failed");
  int64_t* shape = reinterpret_cast<int64_t*>(t + 1);
  int64_t* strides = shape + 3;
  for (int k = 0; k < 3; k++) { shape[k] = b.shape[k]; strides[k] = b.strides[k]; }
  t->dl_tensor.data = b.data;
  t->dl_tensor.device.device_type = 2;  // kDLCUDA
  t->dl_tensor.device.device_id = h->cfg.device;
  t->dl_tensor.ndim = b.ndim;
  t->dl_tensor.dtype.code = (uint8_t)b.dtype_code;
  t->dl_tensor.dtype.bits = (uint8_t)b.dtype_bits;
  t->dl_tensor.dtype.lanes = 1;
  t->dl_tensor.shape = shape;
  t->dl_tensor.strides = strides;
  t->dl_tensor.byte_offset = 0;
  const_cast<gbx_env*>(h)->refs.fetch_add(1, std::memory_order_relaxed);
  t->manager_ctx = const_cast<gbx_env*>(h);
  t->deleter = dl_deleter;
  *out = t;
  return GBX_OK;
}

int gbx_export_state(gbx_env* h, int32_t lo, int32_t hi, const gbx_host_state* o) {
  RET(check_init(h));
  RET(check_range(h, lo, hi));
  if (!o) return fail(GBX_ERR_INVALID, "null out");
  DeviceGuard g(h->cfg.device);
  CK(cudaDeviceSynchronize(), "sync before export");
  const DevState& st = h->st;
  const size_t S = st.S;
  if (o->mem) RET(export_rows(st.mem, MEM_SIZE, lo, hi, o->mem));
  if (o->cart_ram) RET(export_rows(st.cart_ram, h->ram_rows, lo, hi, o->cart_ram));
  if (o->serial) RET(export_rows(st.serial, SERIAL_MAX, lo, hi, o->serial));
  if (o->cart_state) RET(copy_fields(st.cart_state, CS_STRIDE, S, lo, hi, o->cart_state, true));
  if (o->i32) RET(copy_fields(st.i32, I32_COUNT, S, lo, hi, o->i32, true));
  if (o->i64) RET(copy_fields(st.i64, I64_COUNT, S, lo, hi, o->i64, true));
  if (o->u8s) RET(copy_fields(st.u8s, U8_COUNT, S, lo, hi, o->u8s, true));
  if (o->latch) CK(cudaMemcpy(o->latch, st.latch, 9 * SCREEN_H, cudaMemcpyDeviceToHost), "latch copy");
  if (o->obs && hi > lo)
    CK(cudaMemcpy(o->obs, st.obs + (size_t)lo * OBS_DIM, sizeof(float) * OBS_DIM * (hi - lo), cudaMemcpyDeviceToHost),
       "obs copy");
  if (o->reward && hi > lo)
    CK(cudaMemcpy(o->reward, st.reward + lo, sizeof(float) * (hi - lo), cudaMemcpyDeviceToHost), "reward copy");
  return GBX_OK;
}

int gbx_import_state(gbx_env* h, int32_t lo, int32_t hi, const gbx_host_state* in) {
  RET(check_init(h));
  RET(check_range(h, lo, hi));
  if (!in) return fail(GBX_ERR_INVALID, "null in");
  DeviceGuard g(h->cfg.device);
  CK(cudaDeviceSynchronize(), "sync before import");
  const DevState& st = h->st;
  const size_t S = st.S;
  if (in->mem) RET(import_rows(st.mem, MEM_SIZE, lo, hi, in->mem));
  if (in->cart_ram) RET(import_rows(st.cart_ram, h->ram_rows, lo, hi, in->cart_ram));
  if (in->serial) RET(import_rows(st.serial, SERIAL_MAX, lo, hi, in->serial));
  if (in->cart_state) RET(copy_fields(st.cart_state, CS_STRIDE, S, lo, hi, in->cart_state, false));
  if (in->i32) RET(copy_fields(st.i32, I32_COUNT, S, lo, hi, in->i32, false));
  if (in->i64) RET(copy_fields(st.i64, I64_COUNT, S, lo, hi, in->i64, false));
  if (in->u8s) RET(copy_fields(st.u8s, U8_COUNT, S, lo, hi, in->u8s, false));
  if (in->latch) CK(cudaMemcpy(st.latch, in->latch, 9 * SCREEN_H, cudaMemcpyHostToDevice), "latch copy");
  if (in->obs && hi > lo)
    CK(cudaMemcpy(st.obs + (size_t)lo * OBS_DIM, in->obs, sizeof(float) * OBS_DIM * (hi - lo), cudaMemcpyHostToDevice),
       "obs copy");
  if (in->reward && hi > lo)
    CK(cudaMemcpy(st.reward + lo, in->reward, sizeof(float) * (hi - lo), cudaMemcpyHostToDevice), "reward copy");
  CK(cudaDeviceSynchronize(), "sync after import");
  return GBX_OK;
}

int gbx_read_mem(gbx_env* h, int32_t env_idx, int32_t lo, int32_t hi, uint8_t* host_out) {
  RET(check_init(h));
  if (env_idx < 0 || env_idx >= h->st.n)
    return fail(GBX_ERR_RANGE, "env_idx %d out of range [0, %d)", env_idx, h->st.n);
  if (lo < 0 || hi < 0 || lo > MEM_SIZE || hi > MEM_SIZE || lo > hi)
    return fail(GBX_ERR_RANGE, "Invalid memory range: lo=%d hi=%d", lo, hi);
  if (hi == lo) return GBX_OK;
  if (!host_out) return fail(GBX_ERR_INVALID, "null out");
  DeviceGuard g(h->cfg.device);
  CK(cudaDeviceSynchronize(), "sync before read");
  const uint8_t* src = h->st.mem + (size_t)env_idx * MEM_SIZE + lo;
  CK(cudaMemcpy(host_out, src, (size_t)(hi - lo), cudaMemcpyDeviceToHost), "read copy");
  return GBX_OK;
}

int gbx_render_bg_env0(gbx_env* h, uint8_t* out, void* stream) {
  RET(check_init(h));
  DeviceGuard g(h->cfg.device);
  CK(launch_render_bg_env0(h->st, out ? out : h->frame_bg, S_(stream)), "render_bg kernel");
  return GBX_OK;
}

int gbx_set_debug_traps(gbx_env* h, int32_t trap_pc, int32_t trap_rst38, int64_t max_instr, int32_t watch_addr) {
  RET(check_env(h));
  if (max_instr < 0) return fail(GBX_ERR_INVALID, "max_instr must be >= 0, got %lld", (long long)max_instr);
  h->dbg.trap_pc = trap_pc & 0xFFFF;
  h->dbg.trap_rst38 = trap_rst38 ? 1 : 0;
  h->dbg.max_instr = max_instr;
  h->dbg.watch_addr = watch_addr & 0xFFFF;
  return GBX_OK;
}

int gbx_device_status(gbx_env* h, uint32_t* out, int32_t clear) {
  RET(check_env(h));
  if (!out) return fail(GBX_ERR_INVALID, "null out");
  DeviceGuard g(h->cfg.device);
  CK(cudaDeviceSynchronize(), "sync before status");
  CK(cudaMemcpy(out, h->st.status, sizeof(uint32_t), cudaMemcpyDeviceToHost), "status copy");
  if (clear) CK(cudaMemset(h->st.status, 0, sizeof(uint32_t)), "status clear");
  return GBX_OK;
}

}  // extern "C"
