// gbx_layout.h - device-side data layout shared by every kernel of libgbx.
//
// HBM layout (one allocation set per handle; S = SoA row stride, n rounded up
// to a multiple of 128):
//   mem        u8  [N][65536]           env-major: env e's address space is
//                                       one contiguous 64 KiB block, exactly
//                                       the reference's mem view
//                                       (warp_vec.py:799-810)
//   cart_ram   u8  [N][ram_rows]        env-major (ram_rows = max(ram_bytes, 1))
//   serial     u8  [N][1024]            env-major
//   cart_state i32 [20][S]              field-major (SoA)
//   i32        i32 [I32_COUNT][S]       one row per scalar field (SoA)
//   i64        i64 [2][S]               instr_count, cycle_count
//   u8s        u8  [U8_COUNT][S]        joyp_select, serial_overflow, stat_prev
//   latch      u8  [9][144]             env-0 scanline latches
//   obs        f32 [N][32], reward f32 [N]   (reference layout, torch views)
//   pix_packed u8  [N][72][20], pix u8 [N][72][80]
// Env-major byte arrays keep every env's stack, HRAM and IO page in lines of
// its own: an interleaved layout makes the warps of neighbouring envs write
// single bytes of one shared sector, and read-after-write on the stack then
// serialises in L2. The per-env scalars are only touched at the start and end
// of a launch, so they stay SoA; the host API converts them when it exports
// state (the reference keeps them env-major, warp_vec.py:279-497).
#pragma once
#include <stdint.h>

namespace gbx {

constexpr int MEM_SIZE = 65536;
constexpr int CYCLES_PER_FRAME = 70224;
constexpr int CYCLES_PER_LINE = 456;
constexpr int LINES_PER_FRAME = 154;
constexpr int SCREEN_H = 144;
constexpr int ROM_BANK = 0x4000;
constexpr int RAM_BANK = 0x2000;
constexpr int SERIAL_MAX = 1024;
constexpr int OBS_DIM = 32;
constexpr int CS_STRIDE = 20;
constexpr int RTC_CPS = 4194304;
constexpr int PACKED_BYTES = 72 * 20;   // 1440 per env
constexpr int SHADE_BYTES = 72 * 80;    // 5760 per env
constexpr int ROM_SMEM_MAX = 0x8000;    // banks 0-1 staged in shared memory

enum MbcKind { MBC_ROM_ONLY = 0, MBC_MBC1 = 1, MBC_MBC3 = 2 };
enum Stage { STAGE_EMULATE = 0, STAGE_OBS = 1, STAGE_REWARD = 2, STAGE_FULL = 3 };

// cart_state record (src/gbxcule/core/cartridge.py:56-76)
enum CartField {
  CS_MBC_KIND, CS_RAM_ENABLE, CS_ROM_BANK_LO, CS_ROM_BANK_HI, CS_RAM_BANK, CS_BANK_MODE,
  CS_BOOTROM, CS_RTC_SELECT, CS_RTC_LATCH, CS_RTC_S, CS_RTC_M, CS_RTC_H, CS_RTC_DL,
  CS_RTC_DH, CS_RTC_LAST, CS_RTC_LS, CS_RTC_LM, CS_RTC_LH, CS_RTC_LDL, CS_RTC_LDH
};

// i32 SoA rows
enum I32Field {
  F_PC, F_SP, F_A, F_B, F_C, F_D, F_E, F_H, F_L, F_F,
  F_CYCLE_IN_FRAME, F_TRAP_FLAG, F_TRAP_PC, F_TRAP_OPCODE, F_TRAP_KIND,
  F_SERIAL_LEN, F_IME, F_IME_DELAY, F_HALTED, F_DIV_COUNTER, F_TIMER_PREV_IN,
  F_TIMA_RELOAD_PENDING, F_TIMA_RELOAD_DELAY, F_PPU_SCANLINE_CYCLE, F_PPU_LY,
  F_PPU_WINDOW_LINE, F_ACTIONS, I32_COUNT
};
enum I64Field { F_INSTR_COUNT, F_CYCLE_COUNT, I64_COUNT };
enum U8Field { F_JOYP_SELECT, F_SERIAL_OVERFLOW, F_STAT_PREV, U8_COUNT };

// device status bits (OR-ed into DevState::status)
enum StatusBits {
  STATUS_MBC_MISMATCH = 1,   // an env's cart_state mbc_kind differs from the cart's
  STATUS_BAD_ARGS = 2,
};

struct DevState {
  const uint8_t* rom;     // [rom_bytes + 16] shared, read-only (16 zero bytes of padding)
  const uint8_t* boot;    // [256]
  int32_t rom_bytes, rom_bank_count, rom_bank_mask, ram_bank_count;
  int32_t n, S;           // envs, SoA row stride
  int32_t ram_rows;       // cart_ram bytes per env (>= 1)
  int32_t mbc_kind;
  uint8_t* mem;
  uint8_t* cart_ram;
  uint8_t* serial;
  int32_t* cart_state;
  int32_t* i32;
  int64_t* i64;
  uint8_t* u8s;
  uint8_t* latch;
  float* obs;
  float* reward;
  uint32_t* status;
  uint8_t* pix;           // [N][72*80] shade buffer, or null (render_pixels=False)
};

// Debug traps of the reference kernel (cpu_step_builder.py:1320-1393,
// configured from GBXCULE_TRAP_PC / _TRAP_RST38 / _MAX_INSTR / _WATCH_ADDR by
// cpu_step.py:85-105); 0 = off. Trap kinds: 5 pc, 3 RST 38, 4 jump into
// FE00-FFFF, 6 instruction budget, 7 watched byte changed.
struct DebugCfg {
  int32_t trap_pc, trap_rst38, watch_addr;
  int64_t max_instr;
  __host__ __device__ bool active() const { return trap_pc || trap_rst38 || watch_addr || max_instr > 0; }
};

// Device-resident copy of one env (ResetCache, src/gbxcule/core/reset_cache.py:22-64).
struct Snapshot {
  uint8_t* mem;         // [65536]
  uint8_t* cart_ram;    // [ram_bytes] (>= 1)
  uint8_t* serial;      // [1024]
  int32_t* cart_state;  // [20]
  int32_t* i32;         // [I32_COUNT]
  int64_t* i64;         // [I64_COUNT]
  uint8_t* u8s;         // [U8_COUNT]
  uint8_t* pix;         // [72*80] shade image, or null when the batch has no shade buffer
  int32_t ram_bytes;
};

}  // namespace gbx
