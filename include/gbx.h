/*
 * gbx.h - C ABI of libgbx, the B200 (sm_100a) vectorized Game Boy core.
 *
 * One gbx_env is a batch of independent DMG consoles resident on one GPU.
 * Every entry point returns a gbx_status; no exception crosses this boundary.
 * On failure gbx_last_error() returns a message for the calling thread.
 * Device work is enqueued on the caller's stream (a cudaStream_t passed as
 * void*, NULL = legacy default stream) and never synchronises unless the
 * function says so.
 *
 * Each entry point replaces a piece of the reference's vectorized backend
 * (bkase/gbxcule, src/gbxcule/backends/warp_vec.py and
 * src/gbxcule/core/reset_cache.py); the citation is beside each declaration.
 * The Python binding (gbxcule_b200/_lib.py) maps these calls onto the
 * reference's method names and exception types.
 */
#ifndef GBX_H_
#define GBX_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GBX_ABI_VERSION 5

typedef enum {
  GBX_OK = 0,
  GBX_ERR_INVALID = 1,  /* bad argument (maps to ValueError/TypeError)        */
  GBX_ERR_CUDA = 2,     /* CUDA runtime error                                 */
  GBX_ERR_OOM = 3,      /* device allocation failed                           */
  GBX_ERR_STATE = 4,    /* not initialised / wrong order (maps RuntimeError)   */
  GBX_ERR_RANGE = 5     /* index or range out of bounds (maps ValueError)      */
} gbx_status;

/* Post-step body of the step kernel (src/gbxcule/kernels/cpu_step.py:328-341). */
typedef enum {
  GBX_STAGE_EMULATE_ONLY = 0,
  GBX_STAGE_OBS_ONLY = 1,
  GBX_STAGE_REWARD_ONLY = 2,
  GBX_STAGE_FULL_STEP = 3
} gbx_stage;

/* Device buffers exposed for zero-copy views (warp_vec.py:799-901). */
typedef enum {
  GBX_BUF_MEM = 0,            /* u8  [n, 65536]   contiguous        */
  GBX_BUF_PIXELS = 1,         /* u8  [n, 72, 80]  contiguous        */
  GBX_BUF_PIXELS_PACKED = 2,  /* u8  [n, 72, 20]  contiguous        */
  GBX_BUF_OBS = 3,            /* f32 [n, 32]      contiguous        */
  GBX_BUF_REWARD = 4,         /* f32 [n]                            */
  GBX_BUF_CART_RAM = 5,       /* u8  [n, max(ram,1)] contiguous     */
  GBX_BUF_SERIAL = 6,         /* u8  [n, 1024]    contiguous        */
  GBX_BUF_I32 = 7,            /* i32 [GBX_I32_COUNT, n] strides [S, 1] */
  GBX_BUF_I64 = 8,            /* i64 [2, n]       strides [S, 1]    */
  GBX_BUF_U8 = 9,             /* u8  [3, n]       strides [S, 1]    */
  GBX_BUF_CART_STATE = 10,    /* i32 [20, n]      strides [S, 1]    */
  GBX_BUF_LATCH = 11,         /* u8  [9, 144]     env-0 scanline latches */
  GBX_BUF_FRAME_BG = 12,      /* u8  [144, 160]   env-0 frame (gbx_render_bg_env0) */
  GBX_BUF_COUNT = 13
} gbx_buffer_id;

/* Rows of GBX_BUF_I32 (reference field names, warp_vec.py:342-419). */
typedef enum {
  GBX_F_PC, GBX_F_SP, GBX_F_A, GBX_F_B, GBX_F_C, GBX_F_D, GBX_F_E, GBX_F_H, GBX_F_L, GBX_F_F,
  GBX_F_CYCLE_IN_FRAME, GBX_F_TRAP_FLAG, GBX_F_TRAP_PC, GBX_F_TRAP_OPCODE, GBX_F_TRAP_KIND,
  GBX_F_SERIAL_LEN, GBX_F_IME, GBX_F_IME_DELAY, GBX_F_HALTED, GBX_F_DIV_COUNTER,
  GBX_F_TIMER_PREV_IN, GBX_F_TIMA_RELOAD_PENDING, GBX_F_TIMA_RELOAD_DELAY,
  GBX_F_PPU_SCANLINE_CYCLE, GBX_F_PPU_LY, GBX_F_PPU_WINDOW_LINE, GBX_F_ACTIONS,
  GBX_I32_COUNT
} gbx_i32_field;
/* Rows of GBX_BUF_I64 and GBX_BUF_U8. */
typedef enum { GBX_F_INSTR_COUNT, GBX_F_CYCLE_COUNT, GBX_I64_COUNT } gbx_i64_field;
typedef enum { GBX_F_JOYP_SELECT, GBX_F_SERIAL_OVERFLOW, GBX_F_PPU_STAT_PREV, GBX_U8_COUNT } gbx_u8_field;

typedef struct {
  int32_t num_envs;              /* > 0 */
  int32_t device;                /* CUDA ordinal */
  int32_t stage;                 /* gbx_stage */
  int32_t alloc_pixels;          /* allocate GBX_BUF_PIXELS (render_pixels=True) */
  int32_t alloc_pixels_packed;   /* allocate GBX_BUF_PIXELS_PACKED */
} gbx_config;

typedef struct {
  int32_t num_envs, env_stride, device, stage;
  int32_t mbc_kind;              /* 0 ROM only, 1 MBC1, 2 MBC3 */
  int32_t rom_bytes, rom_bank_count, rom_bank_mask, ram_bank_count, ram_bytes;
  int32_t sm_count;              /* SMs of the device */
  int32_t envs_per_warp;         /* K of the latest step launch (see gbx_set_envs_per_warp) */
  int32_t envs_per_warp_tuned;   /* 1 once the launch shape is fixed or the automatic choice is made */
  int32_t dispatch;              /* interpreter of the latest step launch: GBX_DISPATCH_SWITCH or _UNIFORM */
} gbx_info;

/* Step-kernel interpreters (gbx_set_dispatch). */
typedef enum { GBX_DISPATCH_AUTO = 0, GBX_DISPATCH_SWITCH = 1, GBX_DISPATCH_UNIFORM = 2 } gbx_dispatch;

typedef struct {
  void* data;                    /* device pointer */
  int32_t dtype_code;            /* DLPack code: 0 int, 1 uint, 2 float */
  int32_t dtype_bits;
  int32_t ndim;
  int64_t shape[3];
  int64_t strides[3];            /* in elements */
} gbx_buffer_info;

/* Host-side state in the reference's layout for envs [lo, hi): byte arrays
 * env-major ([n][rows]), per-env fields field-major ([fields][n]). Any
 * pointer may be NULL to skip that part. */
typedef struct {
  uint8_t* mem;          /* [n][65536]         */
  uint8_t* cart_ram;     /* [n][ram_bytes]     */
  uint8_t* serial;       /* [n][1024]          */
  int32_t* cart_state;   /* [20][n]            */
  int32_t* i32;          /* [GBX_I32_COUNT][n] */
  int64_t* i64;          /* [GBX_I64_COUNT][n] */
  uint8_t* u8s;          /* [GBX_U8_COUNT][n]  */
  uint8_t* latch;        /* [9][144] (env 0)   */
  float* obs;            /* [n][32]            */
  float* reward;         /* [n]                */
} gbx_host_state;

typedef struct gbx_env gbx_env;
typedef struct gbx_snapshot gbx_snapshot;

/* ABI version of the loaded library (GBX_ABI_VERSION). */
int32_t gbx_abi_version(void);
/* Last error message of the calling thread ("" if none). */
const char* gbx_last_error(void);

/* Create a batch: validates the cartridge header (src/gbxcule/core/cartridge.py:139-187),
 * allocates every device buffer (warp_vec.py:249-497) and uploads ROM + boot ROM.
 * The batch is not initialised until gbx_reset. Replaces WarpVecCudaBackend.__init__
 * (warp_vec.py:1188-1232). */
int gbx_create(const gbx_config* cfg, const uint8_t* rom, size_t rom_len, const uint8_t* boot,
               size_t boot_len, gbx_env** out);
/* Release the caller's ownership of the batch (warp_vec.py:1076-1141). NULL is
 * a no-op. The handle must not be used afterwards. Device buffers are freed
 * when the last owner goes: this call, or the deleter of the last DLPack
 * tensor from gbx_export_dlpack still alive. The free synchronises the whole
 * device (cudaDeviceSynchronize), not only one stream. */
int gbx_destroy(gbx_env* env);
int gbx_get_info(const gbx_env* env, gbx_info* out);

/* Initial state of every env (warp_vec.py:249-497): mem zero with the boot ROM at
 * 0x0000-0x00FF, bank_lo=1, bootrom_enabled=1, joyp_select=0x30, all else zero;
 * then, for the obs/full stages, a zero-frame step that fills obs (:498-512). */
int gbx_reset(gbx_env* env, void* stream);

/* One env-step of every env: frames_to_run frames of emulation, then the stage's
 * post-step body (cpu_step_builder.py:876-1781, launched at warp_vec.py:565-650).
 * actions: device int32[num_envs]; like step_torch (warp_vec.py:1234-1269) no range
 * check is made (indices outside 1..7 press nothing). */
int gbx_step(gbx_env* env, const int32_t* actions, int32_t frames_to_run,
             int32_t release_after_frames, void* stream);

/* Envs per warp K of the step kernel: 1..32 fixes it, 0 = automatic (the
 * default; GBX_ENVS_PER_WARP in the environment fixes it for every handle).
 * No counterpart in the reference, whose Warp launch maps one env per thread
 * with Warp's own block size. K never changes a result, only speed. In
 * automatic mode the handle's first real steps each run with one candidate
 * launch shape, twice per candidate (K: the one that fills one wave of warps
 * on the device, half of it, and 32; interpreter: the switch at each K and
 * the uniform datapath at each K >= 16, unless gbx_set_dispatch fixes it),
 * timed with CUDA events around the launches the caller requested, and
 * later steps use the fastest. Synchronises the device. */
int gbx_set_envs_per_warp(gbx_env* env, int32_t envs_per_warp);

/* Interpreter of the step kernel: GBX_DISPATCH_SWITCH (one switch case per
 * instruction family; fastest when a warp's envs share their PCs or a warp
 * holds few envs), GBX_DISPATCH_UNIFORM (every lane runs one fixed datapath
 * steered by a per-opcode descriptor; fastest for full warps of envs at
 * different PCs) or GBX_DISPATCH_AUTO (the default: the automatic mode of
 * gbx_set_envs_per_warp times both among its candidates; GBX_DISPATCH=switch
 * or =uniform in the environment fixes it for every handle). No counterpart
 * in the reference, whose cpu_step kernel is one if-chain dispatch
 * (src/gbxcule/kernels/cpu_step_builder.py:92-125). Never changes a result,
 * only speed. Synchronises the device. */
int gbx_set_dispatch(gbx_env* env, int32_t dispatch);

/* Snapshot renderer (ppu_render_downsampled.py:207-234 packed, :182-204 unpacked)
 * from current memory. out: device buffer of at least base_offset + n*1440 bytes
 * (packed) or n*5760 (unpacked); NULL renders into the env's own
 * GBX_BUF_PIXELS_PACKED / GBX_BUF_PIXELS. Replaces
 * render_pixels_snapshot_packed_to_torch (warp_vec.py:1293-1352) and
 * render_pixels_snapshot (:727-732). */
int gbx_render_packed(gbx_env* env, uint8_t* out, int64_t base_offset, void* stream);
/* gbx_render_packed plus, in the same pass, the policy input a consumer
 * builds from the packed frame: every pixel as bf16 (shade / 3.0, rounded to
 * nearest even as torch rounds float -> bf16) into `scaled` (device, 16-byte
 * aligned, n*5760*2 bytes), laid out [n][72][80] (layout 0) or as 2x2
 * space-to-depth [n][36][40][4] (layout 1: pixel (y, x) at (y/2, x/2,
 * (y&1)*2 + (x&1)), the input of a stride-2 convolution rewritten as a
 * stride-1 one over 4 channels). Replaces the consumer-side unpack of
 * rl/packed_pixels.py:26-71 followed by the policy's frames / 3.0 (the
 * reference's rollouts run those as separate torch passes). */
int gbx_render_packed_scaled(gbx_env* env, uint8_t* out, int64_t base_offset, void* scaled, int32_t layout,
                             void* stream);
int gbx_render_shades(gbx_env* env, uint8_t* out, void* stream);

/* Capture env env_idx into a device snapshot (ResetCache.from_backend,
 * src/gbxcule/core/reset_cache.py:67-190). Enqueued on stream. */
int gbx_snapshot_create(gbx_env* env, int32_t env_idx, void* stream, gbx_snapshot** out);
/* Free a snapshot. Synchronises the whole device (cudaDeviceSynchronize) first. */
int gbx_snapshot_destroy(gbx_snapshot* snap);
/* Restore every env whose mask byte is non-zero from the snapshot
 * (ResetCache.apply_mask_torch, reset_cache.py:192-307,381-411). mask: device
 * uint8[num_envs]. */
int gbx_masked_restore(gbx_env* env, const gbx_snapshot* snap, const uint8_t* mask, void* stream);

/* Describe a device buffer for a zero-copy view (memory_torch / pixels_torch /
 * pixels_packed_torch, warp_vec.py:799-901). */
int gbx_buffer(const gbx_env* env, int32_t which, gbx_buffer_info* out);
/* Same buffer as a DLPack v0 DLManagedTensor* (written to *out). The tensor
 * owns a reference to the batch (manager_ctx): its memory stays valid until
 * the consumer calls the deleter, even after gbx_destroy. */
int gbx_export_dlpack(const gbx_env* env, int32_t which, void** out);

/* Synchronous copies between device state and host buffers in the reference's
 * layout (see gbx_host_state). Used for get_cpu_state/read_memory/get_cart_state
 * (warp_vec.py:1354-1460) and by state load/parity tooling. */
int gbx_export_state(gbx_env* env, int32_t lo, int32_t hi, const gbx_host_state* out);
int gbx_import_state(gbx_env* env, int32_t lo, int32_t hi, const gbx_host_state* in);
/* Raw device memory bytes [lo, hi) of one env, synchronous (warp_vec.py:1369-1390). */
int gbx_read_mem(gbx_env* env, int32_t env_idx, int32_t lo, int32_t hi, uint8_t* host_out);

/* Device status word (bit 1: an env's cart_state mbc_kind differs from the
 * cartridge's); synchronous. Optionally clears it. */
int gbx_device_status(gbx_env* env, uint32_t* out, int32_t clear);

/* Env 0's 160x144 shade frame from the env-0 scanline latches and env 0's
 * VRAM/OAM (kernels/ppu_step.py:11-176; launched after a step when the
 * reference backend has render_bg=True, warp_vec.py:651-671). out: device
 * u8[144*160], or NULL for the handle's own frame buffer (GBX_BUF_FRAME_BG,
 * zeroed by gbx_reset). Enqueued on stream. */
int gbx_render_bg_env0(gbx_env* env, uint8_t* out, void* stream);

/* Debug traps of the reference kernel (cpu_step_builder.py:1320-1393), the
 * values the reference reads from GBXCULE_TRAP_PC, GBXCULE_TRAP_RST38,
 * GBXCULE_MAX_INSTR and GBXCULE_WATCH_ADDR (cpu_step.py:85-105); 0 turns a
 * check off. Applies to every later gbx_step of the handle; a trapped env
 * stops with trap_flag set and trap_kind 5 (pc), 3 (RST 38 outside 0x0038),
 * 4 (jump into FE00-FFFF), 6 (max_instr instructions in one launch) or 7
 * (watched byte changed). */
int gbx_set_debug_traps(gbx_env* env, int32_t trap_pc, int32_t trap_rst38, int64_t max_instr,
                        int32_t watch_addr);

#ifdef __cplusplus
}
#endif

/* DLPack v0 ABI (public standard, dmlc/dlpack dlpack.h v0.8), declared here so
 * callers need no extra header. */
#ifndef DLPACK_VERSION
typedef struct { int32_t device_type; int32_t device_id; } DLDevice;
typedef struct { uint8_t code; uint8_t bits; uint16_t lanes; } DLDataType;
typedef struct {
  void* data;
  DLDevice device;
  int32_t ndim;
  DLDataType dtype;
  int64_t* shape;
  int64_t* strides;
  uint64_t byte_offset;
} DLTensor;
typedef struct DLManagedTensor {
  DLTensor dl_tensor;
  void* manager_ctx;
  void (*deleter)(struct DLManagedTensor* self);
} DLManagedTensor;
#endif

#endif /* GBX_H_ */
