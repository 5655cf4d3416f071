// gbx_step.cu - the env-step kernel: one SM83 console per thread for the whole
// frame-skip loop.
//
// Semantics follow the reference kernel of bkase/gbxcule
// (src/gbxcule/kernels/cpu_step_builder.py:876-1781 and the instruction
// templates in src/gbxcule/kernels/cpu_templates/), quirks included. The
// structure does not: the reference re-reads and re-writes per-env arrays in
// global memory for every register, IO port and timer field on every
// instruction; here that state lives in registers for the whole launch and
// goes back to HBM once at the end.
//
//  * Memory: address-major, env-minor (gbx_layout.h), so lockstep warps
//    coalesce. Cached IO ports (JOYP, DIV, TIMA, TMA, TAC, IF, LCDC, STAT, LY,
//    LYC, WY, IE) live in registers; every path that touches those addresses
//    (CPU access, OAM DMA source, env-0 latches) goes through the cache.
//  * Fetch: ROM banks 0-1 and the 256-byte boot ROM are staged in shared
//    memory; other banks are read through the read-only path.
//  * Execute: a phased interpreter. A 256-entry decode table (shared memory)
//    gives each opcode a family and a memory-read mode; one read site, one
//    family switch over SM83's regular encoding (registers packed into two
//    u32, indexed by bit-field extract; ALU and CB families branch-free), one
//    write site. A divergent warp executes little distinct code.
//  * Post-instruction work is split. The reference updates the timer, DIV,
//    STAT mode bits, stat_prev, LY and the frame counter after every
//    instruction. Here the common case keeps derived state lazy: STAT's low
//    bits and stat_prev are functions of (LY, scanline cycle, LYC, LCD on);
//    DIV/TIMA advance by an accumulated cycle count that is applied exactly
//    (the reference's edge-stepping timer_tick, which is additive over time)
//    only when an edge or reload is due or a timer port is touched. An
//    instruction that halts, traps, writes LCDC/LY or an RTC register, or
//    takes an interrupt, runs the reference's post-processing verbatim on
//    materialised state (slow_post). Results are bit-identical.
//  * HALT: runs of 4-cycle halted iterations that cannot change anything
//    observable except counters (no line boundary, no timer reload, no frame
//    end) are applied in one batch.
#include <cuda_runtime.h>
#include <limits.h>
#include <stdint.h>
#include <stdlib.h>

#include "gbx_layout.h"

namespace gbx {

// ---------------------------------------------------------------------------
// Decode table
// ---------------------------------------------------------------------------
enum Family : uint8_t {
  FM_NOP, FM_LD16, FM_ST_A_IND, FM_LD_A_IND, FM_INC16, FM_DEC16, FM_INC8, FM_DEC8,
  FM_INCDEC_HL, FM_LD8_IMM, FM_ST_HL_IMM, FM_ROTA, FM_ST_SP16, FM_ADDHL, FM_TRAP,
  FM_JR, FM_JRCC, FM_DAA, FM_CPL, FM_SCF, FM_CCF, FM_LDRR, FM_LDR_HL, FM_STHL_R,
  FM_HALT, FM_ALU_R, FM_ALU_V, FM_RET, FM_POP, FM_JP, FM_JPHL, FM_CALL, FM_PUSH,
  FM_RST, FM_CB, FM_ST_A_IO, FM_LD_A_IO, FM_SPADD, FM_LDSPHL, FM_DI, FM_EI
};
enum ReadMode : uint8_t { RD_NONE, RD_HL, RD_BC, RD_DE, RD_A16, RD_FF_N, RD_FF_C, RD_SP };

// entry = family | read_mode << 8
__host__ __device__ constexpr uint16_t decode_entry(int op) {
  int x = op >> 6, y = (op >> 3) & 7, z = op & 7;
  if (op == 0xCB) return FM_CB;
  if (op == 0x10 || op == 0xD3 || op == 0xDB || op == 0xDD || op == 0xE3 || op == 0xE4 ||
      op == 0xEB || op == 0xEC || op == 0xED || op == 0xF4 || op == 0xFC || op == 0xFD)
    return FM_TRAP;
  if (x == 1) {
    if (op == 0x76) return FM_HALT;
    if (z == 6) return FM_LDR_HL | (RD_HL << 8);
    if (y == 6) return FM_STHL_R;
    return FM_LDRR;
  }
  if (x == 2) return z == 6 ? (FM_ALU_V | (RD_HL << 8)) : FM_ALU_R;
  if (x == 0) {
    switch (z) {
      case 0: return op == 0x00 ? FM_NOP : op == 0x08 ? FM_ST_SP16 : op == 0x18 ? FM_JR : FM_JRCC;
      case 1: return (y & 1) ? FM_ADDHL : FM_LD16;
      case 2:
        if (y & 1) return FM_LD_A_IND | ((op == 0x0A ? RD_BC : op == 0x1A ? RD_DE : RD_HL) << 8);
        return FM_ST_A_IND;
      case 3: return (y & 1) ? FM_DEC16 : FM_INC16;
      case 4: return y == 6 ? (FM_INCDEC_HL | (RD_HL << 8)) : FM_INC8;
      case 5: return y == 6 ? (FM_INCDEC_HL | (RD_HL << 8)) : FM_DEC8;
      case 6: return y == 6 ? FM_ST_HL_IMM : FM_LD8_IMM;
      default:
        switch (y) {
          case 4: return FM_DAA;
          case 5: return FM_CPL;
          case 6: return FM_SCF;
          case 7: return FM_CCF;
          default: return FM_ROTA;
        }
    }
  }
  switch (op) {  // x == 3
    case 0xC0: case 0xC8: case 0xD0: case 0xD8: case 0xC9: case 0xD9:
      return FM_RET | (RD_SP << 8);
    case 0xC1: case 0xD1: case 0xE1: case 0xF1: return FM_POP | (RD_SP << 8);
    case 0xC2: case 0xCA: case 0xD2: case 0xDA: case 0xC3: return FM_JP;
    case 0xE9: return FM_JPHL;
    case 0xC4: case 0xCC: case 0xD4: case 0xDC: case 0xCD: return FM_CALL;
    case 0xC5: case 0xD5: case 0xE5: case 0xF5: return FM_PUSH;
    case 0xE0: case 0xE2: case 0xEA: return FM_ST_A_IO;
    case 0xF0: return FM_LD_A_IO | (RD_FF_N << 8);
    case 0xF2: return FM_LD_A_IO | (RD_FF_C << 8);
    case 0xFA: return FM_LD_A_IO | (RD_A16 << 8);
    case 0xE8: case 0xF8: return FM_SPADD;
    case 0xF9: return FM_LDSPHL;
    case 0xF3: return FM_DI;
    case 0xFB: return FM_EI;
    default: break;
  }
  if (z == 6) return FM_ALU_V;  // ALU A,d8
  return FM_RST;                // z == 7
}

struct DecodeTable {
  uint16_t e[256];
};
__host__ __device__ constexpr DecodeTable make_table() {
  DecodeTable t{};
  for (int i = 0; i < 256; i++) t.e[i] = decode_entry(i);
  return t;
}
__constant__ DecodeTable c_decode = make_table();

// ---------------------------------------------------------------------------
// Per-thread emulator state
// ---------------------------------------------------------------------------
#define FLAGS(z, n, h, c) ((((z) ? 1 : 0) << 7) | (((n) ? 1 : 0) << 6) | (((h) ? 1 : 0) << 5) | (((c) ? 1 : 0) << 4))

// events that send an instruction's post-processing down the exact path
enum Event { EV_FIRST = 1, EV_HALT = 2, EV_TRAP = 4, EV_LCDC = 8, EV_PPU = 16, EV_RTC = 32 };

template <int MBC>
struct Emu {
  // addressing
  uint8_t* mem;          // &st.mem[env]; byte a at mem[a * S]
  uint32_t S;
  const uint8_t* rom_s;  // shared memory: rom[0 .. rom_s_bytes)
  const uint8_t* boot_s; // shared memory: boot ROM
  const uint8_t* rom_g;  // global ROM
  int32_t* cart_state;   // &st.cart_state[env]
  uint8_t* cart_ram;     // &st.cart_ram[env]
  uint8_t* serial;       // &st.serial[env]
  int32_t* i32;          // &st.i32[env]
  uint8_t* u8s;          // &st.u8s[env]
  uint8_t* latch;        // st.latch
  int rom_bank_count, rom_bank_mask, ram_bank_count;
  int rom_s_bytes;
  int is_env0;
  // CPU
  uint32_t bcde, hlxa;   // B C D E | H L - A, high byte first
  int f, pc, sp;
  int ime, ime_delay, halted, ime_mask;
  int trap;
  // cached IO ports (values of mem[FFxx]); stat/div_b/prev_in/stat_prev are
  // exact only while lazy == 0
  int joyp, div_b, tima, tma, tac, iflag, lcdc, stat, ly_b, lyc, wy, ie;
  // timer
  int div, rl_pending, rl_delay, prev_in;
  int t_acc, t_next;     // lazy: cycles not yet applied, cycles to the next edge/reload
  // PPU
  int scan, ly, wl, stat_prev;
  int stat_hi, lcd_on;   // lazy: STAT bits 3-7, LCD on at the last refresh
  // cart
  int ram_en, bank_lo, bank_hi, ram_bank, bank_mode, bootrom, rtc_sel, rtc_latch;
  int bank0_off, bankN_off;   // ROM byte offset of a bank region; -1 when out of range
  int rtc_sub, rtc_s, rtc_m, rtc_h, rtc_dl, rtc_dh, rtc_run;
  // step
  int frames_done, release, action;
  int ev, lazy, lcdc_before;

  // ---- registers -------------------------------------------------------
  __device__ __forceinline__ int A() const { return hlxa & 0xFF; }
  __device__ __forceinline__ void setA(int v) { hlxa = (hlxa & 0xFFFFFF00u) | (uint32_t)(v & 0xFF); }
  __device__ __forceinline__ int HL() const { return hlxa >> 16; }
  __device__ __forceinline__ void setHL(int v) { hlxa = (hlxa & 0xFFFFu) | ((uint32_t)(v & 0xFFFF) << 16); }
  __device__ __forceinline__ int BC() const { return bcde >> 16; }
  __device__ __forceinline__ int DE() const { return bcde & 0xFFFF; }
  __device__ __forceinline__ int C_() const { return (bcde >> 16) & 0xFF; }
  // r8 index: 0 B, 1 C, 2 D, 3 E, 4 H, 5 L, 7 A (6 = (HL), never passed)
  __device__ __forceinline__ int getr(int i) const {
    uint32_t w = (i & 4) ? hlxa : bcde;
    return (w >> ((3 - (i & 3)) * 8)) & 0xFF;
  }
  __device__ __forceinline__ void setr(int i, int v) {
    int sh = (3 - (i & 3)) * 8;
    uint32_t m = ~(0xFFu << sh), val = (uint32_t)(v & 0xFF) << sh;
    if (i & 4) hlxa = (hlxa & m) | val; else bcde = (bcde & m) | val;
  }
  // pair index: 0 BC, 1 DE, 2 HL, 3 SP
  __device__ __forceinline__ int getp(int p) const {
    return p == 0 ? (int)(bcde >> 16) : p == 1 ? (int)(bcde & 0xFFFF) : p == 2 ? (int)(hlxa >> 16) : sp;
  }
  __device__ __forceinline__ void setp(int p, int v) {
    v &= 0xFFFF;
    if (p == 0) bcde = (bcde & 0xFFFFu) | ((uint32_t)v << 16);
    else if (p == 1) bcde = (bcde & 0xFFFF0000u) | (uint32_t)v;
    else if (p == 2) hlxa = (hlxa & 0xFFFFu) | ((uint32_t)v << 16);
    else sp = v;
  }

  // ---- memory -------------------------------------------------------------
  __device__ __forceinline__ uint8_t& M(int a) const { return mem[(size_t)a * S]; }

  __device__ __forceinline__ void update_banks() {
    // cpu_step_builder.py:566-592 (bank selection and clamp_bank)
    int b0 = 0, bn = 1;
    if (MBC == MBC_MBC1) {
      int lo = bank_lo & 0x1F, hi = bank_hi & 3;
      if (bank_mode & 1) b0 = hi << 5;
      bn = (hi << 5) | lo;
      if (bn == 0) bn = 1;
    } else if (MBC == MBC_MBC3) {
      bn = bank_lo & 0x7F;
      if (bn == 0) bn = 1;
    }
    int cnt = rom_bank_count, msk = rom_bank_mask;
    if (cnt <= 0) { b0 = 0; bn = 0; }
    else if (msk >= 0) { b0 &= msk; bn &= msk; }
    else { b0 %= cnt; bn %= cnt; }
    bank0_off = b0 < cnt ? b0 * ROM_BANK : -1;
    bankN_off = bn < cnt ? bn * ROM_BANK - ROM_BANK : -1;
  }

  __device__ __forceinline__ int rom_byte(int idx) const {
    return idx < rom_s_bytes ? rom_s[idx] : __ldg(rom_g + idx);
  }
  __device__ __forceinline__ int rom_read(int a) const {
    if (a < 0x100 && bootrom) return boot_s[a];
    int off = a < 0x4000 ? bank0_off : bankN_off;
    if (off < 0) return 0xFF;
    return rom_byte(off + a);
  }

  // STAT low bits / stat_prev as functions of the PPU position (lazy mode)
  __device__ __forceinline__ int ppu_mode() const {
    return ly >= SCREEN_H ? 1 : scan < 80 ? 2 : scan < 250 ? 3 : 0;
  }
  __device__ __forceinline__ int stat_now() const {
    if (!lazy) return stat;
    return stat_hi | ((ly == lyc) << 2) | (lcd_on ? ppu_mode() : 0);
  }
  __device__ __forceinline__ static int prev_bits(int mode, int coinc) {
    return (mode == 0) | ((mode == 1) << 1) | ((mode == 2) << 2) | (coinc << 3);
  }
  __device__ __forceinline__ int stat_prev_now() const {
    if (!lazy) return stat_prev;
    return lcd_on ? prev_bits(ppu_mode(), ly == lyc) : 0;
  }
  __device__ __forceinline__ int div_byte_now() const {
    return lazy ? (((div + t_acc) >> 8) & 0xFF) : div_b;
  }

  __device__ __forceinline__ int io_read(int a) const {
    switch (a & 0xFF) {
      case 0x00: return joyp;
      case 0x04: return div_byte_now();
      case 0x05: return tima;
      case 0x06: return tma;
      case 0x07: return tac;
      case 0x0F: return iflag;
      case 0x40: return lcdc;
      case 0x41: return stat_now();
      case 0x44: return ly_b;
      case 0x45: return lyc;
      case 0x4A: return wy;
      case 0xFF: return ie;
      default: return M(a);
    }
  }
  // raw mem[] view (no echo remap, no cart mapping): OAM DMA source, latches
  __device__ __forceinline__ int raw_read(int a) const {
    return a >= 0xFF00 ? io_read(a) : M(a);
  }

  __device__ __forceinline__ int ram_index(int a) const {
    // cpu_step_builder.py:633-649; returns -1 for "0xFF / dropped"
    int rb = 0;
    if (MBC == MBC_MBC1) { if (bank_mode & 1) rb = ram_bank & 3; }
    else if (MBC == MBC_MBC3) rb = ram_bank & 3;
    int cnt = ram_bank_count;
    rb = cnt <= 0 ? 0 : rb % cnt;
    int env_bytes = cnt * RAM_BANK;
    if (env_bytes <= 0) return -1;
    int off = rb * RAM_BANK + (a - 0xA000);
    return off < env_bytes ? off : -1;
  }
  __device__ __forceinline__ int rtc_live(int k) const {
    return k == 0 ? rtc_s : k == 1 ? rtc_m : k == 2 ? rtc_h : k == 3 ? rtc_dl : rtc_dh;
  }

  __device__ __forceinline__ int cart_read(int a) const {
    if (ram_bank_count <= 0 || ram_en == 0) return 0xFF;
    if (MBC == MBC_MBC3) {
      int sel = rtc_sel & 0x0F;
      if (sel >= 0x08 && sel <= 0x0C) {
        int k = sel - 8;
        if (!rtc_latch) return rtc_live(k) & 0xFF;
        return cart_state[(size_t)(CS_RTC_LS + k) * S] & 0xFF;
      }
    }
    int off = ram_index(a);
    if (off < 0) return 0xFF;
    return cart_ram[(size_t)off * S];
  }

  __device__ __forceinline__ int read8(int addr) const {
    int a = addr & 0xFFFF;
    if (a < 0x8000) return rom_read(a);
    if (a >= 0xFF00) return io_read(a);
    if (a >= 0xE000 && a < 0xFE00) a -= 0x2000;
    if (a >= 0xA000 && a < 0xC000) return cart_read(a);
    return M(a);
  }

  // ---- timer (cpu_step_builder.py:249-372) ------------------------------------
  __device__ __forceinline__ static int div_bit(int t) {
    int s = t & 3;
    return s == 0 ? 9 : s == 1 ? 3 : s == 2 ? 5 : 7;
  }
  __device__ __forceinline__ static int timer_in(int d, int t) {
    return (t & 4) ? ((d >> div_bit(t)) & 1) : 0;
  }
  __device__ __forceinline__ void tima_inc() {
    int old = tima;
    tima = (tima + 1) & 0xFF;
    if (old == 0xFF) { rl_pending = 1; rl_delay = 4; }
  }
  __device__ __forceinline__ void tima_reload() {
    tima = tma;
    iflag |= 0x04;
    rl_pending = 0;
    rl_delay = 0;
  }
  // the reference's timer_tick, exact
  __device__ void timer_tick(int cycles) {
    if (cycles <= 0) return;
    if (!(tac & 4) && !rl_pending) {
      div = (div + cycles) & 0xFFFF;
    } else {
      int remaining = cycles;
      int d = div & 0xFFFF;
      while (remaining > 0) {
        if (rl_pending && rl_delay <= 0) tima_reload();
        int dt = remaining;
        if (rl_pending && rl_delay < dt) dt = rl_delay;
        int edge = 0;
        if (tac & 4) {
          int period = 1 << (div_bit(tac) + 1);
          int edge_dt = period - (d & (period - 1));
          if (edge_dt < dt) dt = edge_dt;
          edge = dt == edge_dt;
        }
        d = (d + dt) & 0xFFFF;
        if (rl_pending) rl_delay -= dt;
        remaining -= dt;
        if (edge) tima_inc();
        if (rl_pending && rl_delay <= 0) tima_reload();
      }
      div = d;
    }
    div_b = (div >> 8) & 0xFF;
    prev_in = timer_in(div, tac);
  }
  // cycles from now until timer_tick would do more than advance DIV
  __device__ __forceinline__ void calc_t_next() {
    int t = INT_MAX;
    if (rl_pending) t = rl_delay;
    if (tac & 4) {
      int period = 1 << (div_bit(tac) + 1);
      int e = period - (div & (period - 1));
      t = e < t ? e : t;
    }
    t_next = t;
  }
  // apply the accumulated cycles exactly
  __device__ void timer_sync() {
    int c = t_acc;
    t_acc = 0;
    timer_tick(c);
    calc_t_next();
  }

  // ---- MBC3 RTC (:375-419) ---------------------------------------------------
  // Live RTC fields stay in registers. Every tick rewrites them masked, as the
  // reference does, even without a rollover.
  __device__ void rtc_tick(int cycles) {
    if (MBC != MBC_MBC3) return;
    if (cycles <= 0 || (rtc_dh & 0x40)) return;
    int sub = (rtc_sub < 0 ? 0 : rtc_sub) + cycles;
    rtc_s &= 0xFF; rtc_m &= 0x3F; rtc_h &= 0x1F;
    int day = ((rtc_dh & 1) << 8) | (rtc_dl & 0xFF);
    while (sub >= RTC_CPS) {
      sub -= RTC_CPS;
      if (++rtc_s >= 60) {
        rtc_s = 0;
        if (++rtc_m >= 60) {
          rtc_m = 0;
          if (++rtc_h >= 24) {
            rtc_h = 0;
            if (++day >= 512) { day %= 512; rtc_dh |= 0x80; }
          }
        }
      }
    }
    rtc_dl = day & 0xFF;
    rtc_dh = (rtc_dh & 0xC0) | ((day >> 8) & 1);
    rtc_sub = sub;
  }

  // ---- PPU (:422-525 and the advance blocks :988-1082 etc.) ------------------
  __device__ __forceinline__ void latch0(int line) {
    if (!is_env0 || line < 0 || line >= SCREEN_H) return;
    uint8_t* L = latch;
    L[0 * SCREEN_H + line] = (uint8_t)lcdc;
    L[1 * SCREEN_H + line] = M(0xFF43);
    L[2 * SCREEN_H + line] = M(0xFF42);
    L[3 * SCREEN_H + line] = M(0xFF47);
    L[4 * SCREEN_H + line] = M(0xFF4B);
    L[5 * SCREEN_H + line] = (uint8_t)wy;
    L[6 * SCREEN_H + line] = (uint8_t)(wl & 0xFF);
    L[7 * SCREEN_H + line] = M(0xFF48);
    L[8 * SCREEN_H + line] = M(0xFF49);
  }

  // one line boundary: window line, LY, STAT edge IRQ, VBlank, latch.
  // keep = STAT bits 3-7; sp = stat_prev before the line (updated)
  __device__ __forceinline__ void line_step(int l, int keep, int& sp) {
    int prev = ly;
    if (prev < SCREEN_H && (l & 0x20) && prev >= wy) wl++;
    ly = ly + 1 == LINES_PER_FRAME ? 0 : ly + 1;
    if (ly == 0) wl = 0;
    ly_b = ly;
    int mode = ly >= SCREEN_H ? 1 : 0;
    int cur = prev_bits(mode, ly == lyc);
    if ((keep >> 3) & cur & ~(sp & 0xF)) iflag |= 0x02;
    sp = cur;
    if (prev == 143 && ly == 144) iflag |= 0x01;
    if (ly < SCREEN_H) latch0(ly);
  }

  // the reference's advance block, exact (lazy == 0); returns the LCDC it read
  __device__ int ppu_advance(int cycles) {
    int l = lcdc;
    if (!(l & 0x80)) {
      scan = 0; ly = 0; wl = 0; ly_b = 0;
      stat = (stat & 0xF8) | ((lyc == 0) << 2);
      stat_prev = 0;
      return l;
    }
    int total = scan + cycles;
    int lines = total / CYCLES_PER_LINE;
    scan = total - lines * CYCLES_PER_LINE;
    if (lines == 0 && scan == 0) latch0(ly);
    int sp = stat_prev;
    while (lines > 0) {
      line_step(l, stat & 0xF8, sp);
      lines--;
    }
    int mode = ppu_mode();
    int c = ly == lyc;
    stat = (stat & 0xF8) | (c << 2) | mode;
    stat_prev = prev_bits(mode, c);
    return l;
  }

  // lazy advance (lazy == 1, no LCDC/LY write in this instruction)
  __device__ __forceinline__ void ppu_lazy(int cycles) {
    if (!lcd_on) return;
    int total = scan + cycles;
    if (total < CYCLES_PER_LINE) { scan = total; return; }
    int sp = prev_bits(ppu_mode(), ly == lyc);  // stat_prev as of the last refresh
    int lines = total / CYCLES_PER_LINE;
    scan = total - lines * CYCLES_PER_LINE;
    while (lines > 0) {
      line_step(lcdc, stat_hi, sp);
      lines--;
    }
  }

  // ---- lazy <-> exact --------------------------------------------------------
  __device__ void materialize() {
    if (!lazy) return;
    stat = stat_now();
    stat_prev = stat_prev_now();
    lazy = 0;
    int c = t_acc;
    t_acc = 0;
    timer_tick(c);  // no edge/reload is due (t_acc < t_next)
    if (c == 0) { div_b = (div >> 8) & 0xFF; prev_in = timer_in(div, tac); }
  }
  // after an exact post: derived values agree with the state again
  __device__ void delazify() {
    lazy = 1;
    stat_hi = stat & 0xF8;
    lcd_on = (lcdc & 0x80) != 0;
    t_acc = 0;
    calc_t_next();
    ime_mask = ime ? 0x1F : 0;
    rtc_run = (rtc_dh & 0x40) ? 0 : -1;
    ev = 0;
  }

  // ---- writes (:660-873) -----------------------------------------------------
  __device__ __forceinline__ int joyp_value(int sel) const {
    // :196-247
    int pressed = frames_done < release;
    int dpad = 0, btn = 0;
    if (pressed) {
      dpad = action == 4 ? 4 : action == 5 ? 8 : action == 6 ? 2 : action == 7 ? 1 : 0;
      btn = action == 1 ? 1 : action == 2 ? 2 : action == 3 ? 8 : 0;
    }
    int p14 = (sel >> 4) & 1, p15 = (sel >> 5) & 1;
    int v = (sel | 0xCF) & 0xFF;
    if (p14 && p15) v = 0x0F;
    else if (!p14 && p15) v &= 0x0F & ~dpad;
    else if (p14 && !p15) v &= 0x0F & ~btn;
    return v | 0xC0;
  }

  __device__ void write8(int addr, int val) {
    int a = addr & 0xFFFF;
    if (a >= 0xE000 && a < 0xFE00) a -= 0x2000;
    int v8 = val & 0xFF;
    if (a >= 0xFF00) {
      switch (a & 0xFF) {
        case 0x00: {
          int sel = v8 & 0x30;
          u8s[(size_t)F_JOYP_SELECT * S] = (uint8_t)sel;
          joyp = joyp_value(sel);
          return;
        }
        case 0x0F: iflag = v8 & 0x1F; return;
        case 0x02:
          if ((val & 0x80) && (val & 0x01)) {
            int idx = i32[(size_t)F_SERIAL_LEN * S];
            if (idx < SERIAL_MAX) {
              serial[(size_t)idx * S] = M(0xFF01);
              i32[(size_t)F_SERIAL_LEN * S] = idx + 1;
            } else {
              u8s[(size_t)F_SERIAL_OVERFLOW * S] = 1;
            }
            M(0xFF02) = (uint8_t)(val & 0x7F);
            iflag |= 0x08;
          } else {
            M(0xFF02) = (uint8_t)v8;
          }
          return;
        case 0x50:
          if (val != 0) bootrom = 0;
          return;
        case 0x04: case 0x05: case 0x06: case 0x07: {
          if (lazy) timer_sync();
          int reg = a & 0xFF;
          if (reg == 0x05) { tima = v8; }
          else if (reg == 0x06) { tma = v8; }
          else if (reg == 0x04) {
            int pre = timer_in(div & 0xFFFF, tac);
            div_b = 0;
            div = 0;
            int post = timer_in(0, tac);
            prev_in = post;
            if (pre && !post) tima_inc();
          } else {
            int pre = timer_in(div & 0xFFFF, tac);
            int tn = val & 7;
            tac = tn;
            int post = timer_in(div & 0xFFFF, tn);
            prev_in = post;
            if (pre && !post) tima_inc();
          }
          if (lazy) calc_t_next();
          return;
        }
        case 0x46: {
          M(0xFF46) = (uint8_t)v8;
          int src = (val & 0xFF) << 8;
          if (src < 0xFF00) {
            for (int o = 0; o < 160; o++) M(0xFE00 + o) = M((src + o) & 0xFFFF);
          } else {
            for (int o = 0; o < 160; o++) M(0xFE00 + o) = (uint8_t)raw_read(src + o);
          }
          return;
        }
        case 0xFF: ie = v8 & 0x1F; return;
        case 0x40:
          if (!(ev & EV_LCDC)) lcdc_before = lcdc;
          lcdc = v8;
          ev |= EV_LCDC;
          return;
        case 0x41: stat = v8; stat_hi = v8 & 0xF8; return;
        case 0x44: ly_b = v8; ev |= EV_PPU; return;
        case 0x45:
          // stat_prev of the last refresh was computed with the old LYC
          if (lazy) materialize();
          lyc = v8;
          ev |= EV_PPU;
          return;
        case 0x4A: wy = v8; return;
        default: M(a) = (uint8_t)v8; return;
      }
    }
    if (a >= 0xA000 && a < 0xC000) {
      if (ram_bank_count <= 0 || ram_en == 0) return;
      if (MBC == MBC_MBC3) {
        int sel = rtc_sel & 0x0F;
        if (sel >= 0x08 && sel <= 0x0C) {
          switch (sel) {
            case 0x08: rtc_s = v8; break;
            case 0x09: rtc_m = v8; break;
            case 0x0A: rtc_h = v8; break;
            case 0x0B: rtc_dl = v8; break;
            default: rtc_dh = v8; break;
          }
          ev |= EV_RTC;
          return;
        }
      }
      int off = ram_index(a);
      if (off >= 0) cart_ram[(size_t)off * S] = (uint8_t)v8;
      return;
    }
    if (a < 0x8000) {
      if (MBC == MBC_MBC1) {
        if (a < 0x2000) ram_en = (val & 0x0F) == 0x0A;
        else if (a < 0x4000) { int b = val & 0x1F; bank_lo = b ? b : 1; }
        else if (a < 0x6000) { bank_hi = val & 3; ram_bank = val & 3; }
        else bank_mode = val & 1;
        update_banks();
      } else if (MBC == MBC_MBC3) {
        if (a < 0x2000) ram_en = (val & 0x0F) == 0x0A;
        else if (a < 0x4000) { int b = val & 0x7F; bank_lo = b ? b : 1; update_banks(); }
        else if (a < 0x6000) { int sel = val & 0x0F; rtc_sel = sel; if (sel <= 3) ram_bank = sel; }
        else {
          if (val == 0) rtc_latch = 0;
          else if (val == 1 && rtc_latch == 0) {
            for (int k = 0; k < 5; k++) cart_state[(size_t)(CS_RTC_LS + k) * S] = rtc_live(k);
            rtc_latch = 1;
          }
        }
      }
      return;
    }
    M(a) = (uint8_t)v8;
  }

  // ---- ALU (alu.py), branch-free over the 8 kinds ----------------------------
  __device__ __forceinline__ void alu(int kind, int v) {
    const int a = A();
    const int cin = (kind == 1 || kind == 3) ? ((f >> 4) & 1) : 0;
    const bool sub = kind == 2 || kind == 3 || kind == 7;
    const int lo = sub ? (a & 0xF) - (v & 0xF) - cin : (a & 0xF) + (v & 0xF) + cin;
    const int full = sub ? a - v - cin : a + v + cin;
    const int h = sub ? lo < 0 : lo > 0xF;
    const int c = sub ? full < 0 : full > 0xFF;
    const bool logic = kind >= 4 && kind <= 6;
    const int lres = kind == 4 ? (a & v) : kind == 5 ? (a ^ v) : (a | v);
    const int res = (logic ? lres : full) & 0xFF;
    const int fl = logic ? (kind == 4 ? 0x20 : 0) : ((sub << 6) | (h << 5) | (c << 4));
    f = ((res == 0) << 7) | fl;
    if (kind != 7) setA(res);
  }
  __device__ __forceinline__ bool cond(int cc) const {
    int bit = (cc & 2) ? ((f >> 4) & 1) : ((f >> 7) & 1);
    return (cc & 1) ? bit : !bit;
  }
};

__device__ __forceinline__ int sign8(int v) { return v >= 128 ? v - 256 : v; }

// ---------------------------------------------------------------------------
// Post-processing, exact (the reference's per-instruction tail)
// ---------------------------------------------------------------------------
// stage 0: nothing applied yet for this instruction's `cyc` cycles.
// stage 1: timer and PPU already advanced lazily by `cyc` (the fast path found
//          a pending interrupt).
template <int MBC>
__device__ void slow_post(Emu<MBC>& s, int cyc, int opcode, int pc_before, int stage, int frames_to_run,
                          int& cycle_frame, long long& cyc_total) {
  const int lcdc_prev = ((s.ev & EV_LCDC) ? s.lcdc_before : s.lcdc) & 0x80;
  s.materialize();
  int lcdc_now;
  if (stage == 0) {
    s.timer_tick(cyc);
    if (s.ime_delay) { s.ime = 1; s.ime_delay = 0; }
    lcdc_now = s.ppu_advance(cyc);
  } else {
    lcdc_now = s.lcdc;
  }
  const int pending = s.ie & s.iflag & 0x1F;
  int svc = 0;
  if (pending) {
    if (s.halted) s.halted = 0;
    if (s.ime) {
      int bit = pending & (-pending);  // lowest set bit = highest priority
      int vector = 0x40 + 8 * (31 - __clz(bit));
      s.ime = 0;
      s.iflag &= 0xFF ^ bit;
      int ret = s.pc;
      s.sp = (s.sp - 1) & 0xFFFF;
      s.write8(s.sp, ret >> 8);
      s.sp = (s.sp - 1) & 0xFFFF;
      s.write8(s.sp, ret & 0xFF);
      s.pc = vector;
      svc = 20;
      s.timer_tick(20);
      lcdc_now = s.ppu_advance(20);
    }
  }
  const int total = cyc + svc;
  s.rtc_tick(total);
  cyc_total += total;
  cycle_frame += total;
  // frame accounting (:1706-1758)
  if (lcdc_prev && !(lcdc_now & 0x80)) {
    int tail = total;
    if (opcode == 0xE0 && (s.read8((pc_before + 1) & 0xFFFF) & 0xFF) == 0x40 && cyc >= 4) tail = total - 4;
    cycle_frame = tail;
    s.frames_done++;
  } else if (!lcdc_prev && (lcdc_now & 0x80)) {
    s.scan = 0; s.ly = 0; s.wl = 0; s.ly_b = 0;
    s.stat = (s.stat & 0xF8) | ((s.lyc == 0) << 2) | 2;
    s.stat_prev = (1 << 2) | ((s.lyc == 0) << 3);
    cycle_frame = 0;
    s.frames_done++;
  } else {
    while (cycle_frame >= CYCLES_PER_FRAME) {
      cycle_frame -= CYCLES_PER_FRAME;
      s.frames_done++;
      if (s.frames_done >= frames_to_run) break;
    }
  }
  s.delazify();
}

// One halted iteration (:976-1300), or a batch of them that no event can
// interrupt. Exact state in and out.
template <int MBC>
__device__ void halted_step(Emu<MBC>& s, int frames_to_run, int& cycle_frame, long long& cyc_total) {
  const int lcdc_prev = s.lcdc & 0x80;
  int k = 1;
  const int pending0 = s.ie & s.iflag & 0x1F;
  if (pending0 == 0 && cycle_frame < CYCLES_PER_FRAME) {
    int kmax = (CYCLES_PER_FRAME - cycle_frame + 3) >> 2;  // iteration that ends the frame
    if (s.lcdc & 0x80) {
      int kl = (CYCLES_PER_LINE - s.scan + 3) >> 2;        // iteration that crosses a line
      kmax = kl < kmax ? kl : kmax;
    }
    if ((s.tac & 4) || s.rl_pending) {
      int t;
      if (s.rl_pending) {
        t = s.rl_delay;
      } else {
        int period = 1 << (Emu<MBC>::div_bit(s.tac) + 1);
        t = period - (s.div & (period - 1)) + (0xFF - s.tima) * period + 4;
      }
      int kt = t <= 0 ? 1 : (t + 3) >> 2;                  // iteration of the next TIMA reload
      kmax = kt < kmax ? kt : kmax;
    }
    k = kmax - 1;
    if (k < 1) k = 1;
  }
  const int cycles = 4 * k;
  s.timer_tick(cycles);
  int lcdc_now = s.ppu_advance(cycles);
  const int pending = s.ie & s.iflag & 0x1F;
  int svc = 0;
  if (pending) {
    s.halted = 0;
    if (s.ime) {
      int bit = pending & (-pending);
      int vector = 0x40 + 8 * (31 - __clz(bit));
      s.ime = 0;
      s.iflag &= 0xFF ^ bit;
      int ret = s.pc;
      s.sp = (s.sp - 1) & 0xFFFF;
      s.write8(s.sp, ret >> 8);
      s.sp = (s.sp - 1) & 0xFFFF;
      s.write8(s.sp, ret & 0xFF);
      s.pc = vector;
      svc = 20;
      s.timer_tick(20);
      lcdc_now = s.ppu_advance(20);
    } else {
      s.pc = (s.pc + 1) & 0xFFFF;  // :1181-1183
    }
  }
  const int total = cycles + svc;
  s.rtc_tick(total);
  cyc_total += total;
  cycle_frame += total;
  if (lcdc_prev && !(lcdc_now & 0x80)) {
    cycle_frame = 0;
    s.frames_done++;
    return;
  }
  while (cycle_frame >= CYCLES_PER_FRAME) {
    cycle_frame -= CYCLES_PER_FRAME;
    s.frames_done++;
    if (s.frames_done >= frames_to_run) break;
  }
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
// K = envs per warp: lane l < K of global warp w runs env w*K + l. Small K
// spreads few envs over many warps (no divergence, more latency hiding);
// K = 32 packs a full warp (shared issue slots when envs run in lockstep).
// REGCAP = 1 caps registers so 4 blocks of 256 threads fit per SM.
template <int MBC, int REGCAP>
__global__ void __launch_bounds__(256, REGCAP ? 4 : 1)
    gb_step_kernel(DevState st, const int32_t* __restrict__ actions, int frames_to_run, int release_after_frames,
                   int stage, int K) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint16_t* dec_s = reinterpret_cast<uint16_t*>(smem);
  uint8_t* boot_s = smem + 512;
  uint8_t* rom_s = smem + 768;
  const int rom_s_bytes = st.rom_bytes < ROM_SMEM_MAX ? st.rom_bytes : ROM_SMEM_MAX;
  {
    const uint4* src = reinterpret_cast<const uint4*>(st.rom);
    uint4* dst = reinterpret_cast<uint4*>(rom_s);
    for (int k = threadIdx.x; k < rom_s_bytes / 16; k += blockDim.x) dst[k] = __ldg(src + k);
    for (int k = threadIdx.x; k < 256; k += blockDim.x) {
      boot_s[k] = st.boot[k];
      dec_s[k] = c_decode.e[k];
    }
  }
  __syncthreads();

  const int lane = threadIdx.x & 31;
  if (lane >= K) return;
  const int env = ((blockIdx.x * blockDim.x + threadIdx.x) >> 5) * K + lane;
  if (env >= st.n) return;
  const size_t S = (size_t)st.S;

  Emu<MBC> s;
  s.mem = st.mem + env;
  s.S = st.S;
  s.rom_s = rom_s;
  s.boot_s = boot_s;
  s.rom_g = st.rom;
  s.cart_state = st.cart_state + env;
  s.cart_ram = st.cart_ram + env;
  s.serial = st.serial + env;
  s.i32 = st.i32 + env;
  s.u8s = st.u8s + env;
  s.latch = st.latch;
  s.rom_bank_count = st.rom_bank_count;
  s.rom_bank_mask = st.rom_bank_mask;
  s.ram_bank_count = st.ram_bank_count;
  s.rom_s_bytes = rom_s_bytes;
  s.is_env0 = env == 0;

  const int32_t* I = st.i32 + env;
  auto ld = [&](int fld) { return I[(size_t)fld * S]; };
  s.pc = ld(F_PC) & 0xFFFF;
  s.sp = ld(F_SP) & 0xFFFF;
  s.bcde = ((uint32_t)(ld(F_B) & 0xFF) << 24) | ((uint32_t)(ld(F_C) & 0xFF) << 16) |
           ((uint32_t)(ld(F_D) & 0xFF) << 8) | (uint32_t)(ld(F_E) & 0xFF);
  s.hlxa = ((uint32_t)(ld(F_H) & 0xFF) << 24) | ((uint32_t)(ld(F_L) & 0xFF) << 16) | (uint32_t)(ld(F_A) & 0xFF);
  s.f = ld(F_F) & 0xF0;
  int cycle_frame = ld(F_CYCLE_IN_FRAME);
  s.trap = ld(F_TRAP_FLAG);
  s.ime = ld(F_IME);
  s.ime_delay = ld(F_IME_DELAY);
  s.halted = ld(F_HALTED);
  s.div = ld(F_DIV_COUNTER);
  s.prev_in = ld(F_TIMER_PREV_IN);
  s.rl_pending = ld(F_TIMA_RELOAD_PENDING);
  s.rl_delay = ld(F_TIMA_RELOAD_DELAY);
  s.scan = ld(F_PPU_SCANLINE_CYCLE);
  s.ly = ld(F_PPU_LY);
  s.wl = ld(F_PPU_WINDOW_LINE);
  s.stat_prev = st.u8s[(size_t)F_STAT_PREV * S + env];
  long long instr = st.i64[(size_t)F_INSTR_COUNT * S + env];
  long long cyc_total = st.i64[(size_t)F_CYCLE_COUNT * S + env];

  s.joyp = s.M(0xFF00); s.div_b = s.M(0xFF04); s.tima = s.M(0xFF05); s.tma = s.M(0xFF06);
  s.tac = s.M(0xFF07); s.iflag = s.M(0xFF0F); s.lcdc = s.M(0xFF40); s.stat = s.M(0xFF41);
  s.ly_b = s.M(0xFF44); s.lyc = s.M(0xFF45); s.wy = s.M(0xFF4A); s.ie = s.M(0xFFFF);

  const int32_t* CSp = st.cart_state + env;
  if (CSp[(size_t)CS_MBC_KIND * S] != st.mbc_kind) atomicOr(st.status, STATUS_MBC_MISMATCH);
  s.ram_en = CSp[(size_t)CS_RAM_ENABLE * S];
  s.bank_lo = CSp[(size_t)CS_ROM_BANK_LO * S];
  s.bank_hi = CSp[(size_t)CS_ROM_BANK_HI * S];
  s.ram_bank = CSp[(size_t)CS_RAM_BANK * S];
  s.bank_mode = CSp[(size_t)CS_BANK_MODE * S];
  s.bootrom = CSp[(size_t)CS_BOOTROM * S];
  s.rtc_sel = CSp[(size_t)CS_RTC_SELECT * S];
  s.rtc_latch = CSp[(size_t)CS_RTC_LATCH * S];
  s.rtc_s = CSp[(size_t)CS_RTC_S * S];
  s.rtc_m = CSp[(size_t)CS_RTC_M * S];
  s.rtc_h = CSp[(size_t)CS_RTC_H * S];
  s.rtc_dl = CSp[(size_t)CS_RTC_DL * S];
  s.rtc_dh = CSp[(size_t)CS_RTC_DH * S];
  s.rtc_sub = CSp[(size_t)CS_RTC_LAST * S];
  s.update_banks();

  s.action = actions[env];
  s.release = release_after_frames;
  s.frames_done = 0;
  // derived state is exact until the first exact post-processing
  s.lazy = 0;
  s.ev = EV_FIRST;
  s.t_acc = 0;
  s.t_next = INT_MAX;
  s.stat_hi = s.stat & 0xF8;
  s.lcd_on = 0;
  s.ime_mask = 0;
  s.rtc_run = 0;
  s.lcdc_before = s.lcdc;

  const uint16_t* dec = dec_s;

  while (s.frames_done < frames_to_run) {
    if (s.trap) break;
    if (s.halted) {
      s.materialize();
      const int first = s.ev & EV_FIRST;
      halted_step(s, frames_to_run, cycle_frame, cyc_total);
      s.delazify();
      s.ev = first;
      continue;
    }
    // ---- fetch ----
    const int pc_before = s.pc;
    int opcode, imm8, imm16;
    {
      const int pc = s.pc;
      const int off = (pc & 0x4000) ? s.bankN_off : s.bank0_off;
      // fast path: three bytes inside one ROM bank region, boot ROM not mapped there
      if (pc < 0x8000 && (pc & 0x3FFF) < 0x3FFE && off >= 0 && (pc >= 0x100 || !s.bootrom)) {
        const int idx = off + pc;
        if (idx + 2 < s.rom_s_bytes) {
          opcode = s.rom_s[idx]; imm8 = s.rom_s[idx + 1]; imm16 = imm8 | (s.rom_s[idx + 2] << 8);
        } else {
          opcode = __ldg(s.rom_g + idx); imm8 = __ldg(s.rom_g + idx + 1);
          imm16 = imm8 | (__ldg(s.rom_g + idx + 2) << 8);
        }
      } else {
        opcode = s.read8(pc);
        imm8 = s.read8(pc + 1);
        imm16 = imm8 | (s.read8(pc + 2) << 8);
      }
    }
    const int e = dec[opcode];
    const int fam = e & 0xFF;
    int rmode = e >> 8;
    if (fam == FM_CB && (imm8 & 7) == 6) rmode = RD_HL;
    // ---- memory reads ----
    int v1 = 0, v2 = 0;
    if (rmode != RD_NONE) {
      int ra;
      switch (rmode) {
        case RD_HL: ra = s.HL(); break;
        case RD_BC: ra = s.BC(); break;
        case RD_DE: ra = s.DE(); break;
        case RD_A16: ra = imm16; break;
        case RD_FF_N: ra = 0xFF00 | imm8; break;
        case RD_FF_C: ra = 0xFF00 | s.C_(); break;
        default: ra = s.sp; break;
      }
      v1 = s.read8(ra);
      if (rmode == RD_SP) v2 = s.read8((ra + 1) & 0xFFFF);
    }
    // ---- execute ----
    int pc = s.pc;
    int cyc = 4;
    int nw = 0, wa0 = 0, wv0 = 0, wa1 = 0, wv1 = 0;
    const int y = (opcode >> 3) & 7, z = opcode & 7;
    switch (fam) {
      case FM_NOP: pc += 1; break;
      case FM_LD16: s.setp((opcode >> 4) & 3, imm16); pc += 3; cyc = 12; break;
      case FM_ST_A_IND: {
        int p = (opcode >> 4) & 3;  // 0 BC, 1 DE, 2 HL+, 3 HL-
        int ad = p == 0 ? s.BC() : p == 1 ? s.DE() : s.HL();
        nw = 1; wa0 = ad; wv0 = s.A();
        if (p >= 2) s.setHL(p == 2 ? ad + 1 : ad - 1);
        pc += 1; cyc = 8; break;
      }
      case FM_LD_A_IND: {
        int p = (opcode >> 4) & 3;
        s.setA(v1);
        if (p >= 2) { int hl = s.HL(); s.setHL(p == 2 ? hl + 1 : hl - 1); }
        pc += 1; cyc = 8; break;
      }
      case FM_INC16: { int p = (opcode >> 4) & 3; s.setp(p, s.getp(p) + 1); pc += 1; cyc = 8; break; }
      case FM_DEC16: { int p = (opcode >> 4) & 3; s.setp(p, s.getp(p) - 1); pc += 1; cyc = 8; break; }
      case FM_INC8: {
        int old = s.getr(y), v = (old + 1) & 0xFF;
        s.setr(y, v);
        s.f = FLAGS(v == 0, 0, (old & 0xF) == 0xF, (s.f >> 4) & 1);
        pc += 1; break;
      }
      case FM_DEC8: {
        int old = s.getr(y), v = (old - 1) & 0xFF;
        s.setr(y, v);
        s.f = FLAGS(v == 0, 1, (old & 0xF) == 0, (s.f >> 4) & 1);
        pc += 1; break;
      }
      case FM_INCDEC_HL: {
        const int old = v1, dec1 = z == 5;
        const int v = (dec1 ? old - 1 : old + 1) & 0xFF;
        const int h = dec1 ? (old & 0xF) == 0 : (old & 0xF) == 0xF;
        s.f = FLAGS(v == 0, dec1, h, (s.f >> 4) & 1);
        nw = 1; wa0 = s.HL(); wv0 = v;
        pc += 1; cyc = 12; break;
      }
      case FM_LD8_IMM: s.setr(y, imm8); pc += 2; cyc = 8; break;
      case FM_ST_HL_IMM: nw = 1; wa0 = s.HL(); wv0 = imm8; pc += 2; cyc = 12; break;
      case FM_ROTA: {
        const int a = s.A(), oc = (s.f >> 4) & 1;
        const int right = y & 1, thru = y >> 1;
        const int c = right ? (a & 1) : ((a >> 7) & 1);
        const int in = thru ? oc : c;
        const int r = right ? ((a >> 1) | (in << 7)) : (((a << 1) & 0xFF) | in);
        s.setA(r); s.f = FLAGS(0, 0, 0, c);
        pc += 1; break;
      }
      case FM_ST_SP16:
        nw = 2; wa0 = imm16; wv0 = s.sp & 0xFF; wa1 = (imm16 + 1) & 0xFFFF; wv1 = (s.sp >> 8) & 0xFF;
        pc += 3; cyc = 20; break;
      case FM_ADDHL: {
        int p = (opcode >> 4) & 3;
        int hl = s.HL(), rr = s.getp(p), sum = hl + rr;
        s.f = FLAGS((s.f >> 7) & 1, 0, ((hl & 0xFFF) + (rr & 0xFFF)) > 0xFFF, sum > 0xFFFF);
        s.setHL(sum);
        pc += 1; cyc = 8; break;
      }
      case FM_JR: pc = pc + 2 + sign8(imm8); cyc = 12; break;
      case FM_JRCC: {
        const bool t = s.cond(y);
        pc = pc + 2 + (t ? sign8(imm8) : 0);
        cyc = t ? 12 : 8;
        break;
      }
      case FM_DAA: {
        int a = s.A(), n = (s.f >> 6) & 1, h = (s.f >> 5) & 1, c = (s.f >> 4) & 1, adj = 0, carry = c;
        if (!n) {
          if (h || (a & 0xF) > 9) adj |= 0x06;
          if (c || a > 0x99) { adj |= 0x60; carry = 1; }
          a = (a + adj) & 0xFF;
        } else {
          if (h) adj |= 0x06;
          if (c) adj |= 0x60;
          a = (a - adj) & 0xFF;
        }
        s.f = FLAGS(a == 0, n, 0, carry); s.setA(a);
        pc += 1; break;
      }
      case FM_CPL: s.setA(s.A() ^ 0xFF); s.f = FLAGS((s.f >> 7) & 1, 1, 1, (s.f >> 4) & 1); pc += 1; break;
      case FM_SCF: s.f = FLAGS((s.f >> 7) & 1, 0, 0, 1); pc += 1; break;
      case FM_CCF: s.f = FLAGS((s.f >> 7) & 1, 0, 0, !((s.f >> 4) & 1)); pc += 1; break;
      case FM_LDRR: s.setr(y, s.getr(z)); pc += 1; break;
      case FM_LDR_HL: s.setr(y, v1); pc += 1; cyc = 8; break;
      case FM_STHL_R: nw = 1; wa0 = s.HL(); wv0 = s.getr(z); pc += 1; cyc = 8; break;
      case FM_HALT: s.halted = 1; s.ev |= EV_HALT; pc += 1; break;
      case FM_ALU_R: s.alu(y, s.getr(z)); pc += 1; break;
      case FM_ALU_V: {
        const bool hl = rmode == RD_HL;
        s.alu(y, hl ? v1 : imm8);
        pc += hl ? 1 : 2;
        cyc = 8; break;
      }
      case FM_RET:
        if (opcode == 0xC9 || opcode == 0xD9 || s.cond(y)) {
          pc = v1 | (v2 << 8);
          s.sp = (s.sp + 2) & 0xFFFF;
          if (opcode == 0xD9) { s.ime = 1; s.ime_delay = 0; s.ime_mask = 0x1F; }
          cyc = (opcode & 1) ? 16 : 20;
        } else {
          pc += 1; cyc = 8;
        }
        break;
      case FM_POP: {
        int p = (opcode >> 4) & 3;
        if (p == 3) { s.setA(v2); s.f = v1 & 0xF0; }
        else s.setp(p, v1 | (v2 << 8));
        s.sp = (s.sp + 2) & 0xFFFF;
        pc += 1; cyc = 12; break;
      }
      case FM_JP: {
        const bool t = opcode == 0xC3 || s.cond(y);
        pc = t ? imm16 : pc + 3;
        cyc = t ? 16 : 12;
        break;
      }
      case FM_JPHL: pc = s.HL(); break;
      case FM_CALL:
        if (opcode == 0xCD || s.cond(y)) {
          int ret = (pc + 3) & 0xFFFF;
          nw = 2; wa0 = (s.sp - 1) & 0xFFFF; wv0 = ret >> 8; wa1 = (s.sp - 2) & 0xFFFF; wv1 = ret & 0xFF;
          s.sp = (s.sp - 2) & 0xFFFF;
          pc = imm16; cyc = 24;
        } else {
          pc += 3; cyc = 12;
        }
        break;
      case FM_PUSH: {
        int p = (opcode >> 4) & 3;
        int v = p == 3 ? ((s.A() << 8) | (s.f & 0xF0)) : s.getp(p);
        nw = 2; wa0 = (s.sp - 1) & 0xFFFF; wv0 = v >> 8; wa1 = (s.sp - 2) & 0xFFFF; wv1 = v & 0xFF;
        s.sp = (s.sp - 2) & 0xFFFF;
        pc += 1; cyc = 16; break;
      }
      case FM_RST: {
        int ret = (pc + 1) & 0xFFFF;
        nw = 2; wa0 = (s.sp - 1) & 0xFFFF; wv0 = ret >> 8; wa1 = (s.sp - 2) & 0xFFFF; wv1 = ret & 0xFF;
        s.sp = (s.sp - 2) & 0xFFFF;
        pc = opcode & 0x38; cyc = 16; break;
      }
      case FM_CB: {
        // bitops.py: all 256 CB ops, branch-free over the group
        const int cb = imm8, cz = cb & 7, cy = (cb >> 3) & 7, grp = cb >> 6;
        const bool hl = cz == 6;
        const int v = hl ? v1 : s.getr(cz);
        const int oc = (s.f >> 4) & 1;
        const int right = cy & 1;
        const int lin = cy == 0 ? (v >> 7) & 1 : cy == 2 ? oc : 0;
        const int rin = cy == 1 ? (v & 1) << 7 : cy == 3 ? oc << 7 : cy == 5 ? (v & 0x80) : 0;
        const int sh = cy == 6 ? (((v & 0xF) << 4) | (v >> 4)) : right ? ((v >> 1) | rin) : (((v << 1) & 0xFF) | lin);
        const int shc = cy == 6 ? 0 : right ? (v & 1) : ((v >> 7) & 1);
        const int mask = 1 << cy;
        const int res = grp == 0 ? sh : grp == 2 ? (v & ~mask) : (v | mask);
        if (grp == 0) s.f = FLAGS(res == 0, 0, 0, shc);
        if (grp == 1) s.f = FLAGS((v & mask) == 0, 0, 1, oc);
        pc += 2;
        if (grp == 1) { cyc = hl ? 12 : 8; break; }
        if (hl) { nw = 1; wa0 = s.HL(); wv0 = res; cyc = 16; }
        else { s.setr(cz, res); cyc = 8; }
        break;
      }
      case FM_ST_A_IO:
        nw = 1; wv0 = s.A();
        if (opcode == 0xE0) { wa0 = 0xFF00 | imm8; pc += 2; cyc = 12; }
        else if (opcode == 0xE2) { wa0 = 0xFF00 | s.C_(); pc += 1; cyc = 8; }
        else { wa0 = imm16; pc += 3; cyc = 16; }
        break;
      case FM_LD_A_IO:
        s.setA(v1);
        if (opcode == 0xF0) { pc += 2; cyc = 12; }
        else if (opcode == 0xF2) { pc += 1; cyc = 8; }
        else { pc += 3; cyc = 16; }
        break;
      case FM_SPADD: {
        int ou = imm8, res = (s.sp + sign8(imm8)) & 0xFFFF;
        s.f = FLAGS(0, 0, ((s.sp & 0xF) + (ou & 0xF)) > 0xF, ((s.sp & 0xFF) + ou) > 0xFF);
        if (opcode == 0xE8) { s.sp = res; cyc = 16; }
        else { s.setHL(res); cyc = 12; }
        pc += 2; break;
      }
      case FM_LDSPHL: s.sp = s.HL(); pc += 1; cyc = 8; break;
      case FM_DI: s.ime = 0; s.ime_delay = 0; s.ime_mask = 0; pc += 1; break;
      case FM_EI: s.ime = 1; s.ime_delay = 0; s.ime_mask = 0x1F; pc += 1; break;
      default:  // FM_TRAP (misc.py:42-56)
        s.trap = 1;
        s.ev |= EV_TRAP;
        st.i32[(size_t)F_TRAP_PC * S + env] = pc & 0xFFFF;
        st.i32[(size_t)F_TRAP_OPCODE * S + env] = opcode & 0xFF;
        st.i32[(size_t)F_TRAP_KIND * S + env] = 1;
        cyc = 0;
        break;
    }
    s.pc = pc & 0xFFFF;
    // ---- memory writes ----
    if (nw) {
      s.write8(wa0, wv0);
      if (nw == 2) s.write8(wa1, wv1);
    }
    // ---- post-processing ----
    if (s.ev) {
      if (s.trap) break;
      instr++;
      slow_post(s, cyc, opcode, pc_before, 0, frames_to_run, cycle_frame, cyc_total);
      continue;
    }
    instr++;
    s.t_acc += cyc;
    if (s.t_acc >= s.t_next) s.timer_sync();
    s.ppu_lazy(cyc);
    if (s.ie & s.iflag & s.ime_mask) {
      slow_post(s, cyc, opcode, pc_before, 1, frames_to_run, cycle_frame, cyc_total);
      continue;
    }
    if (MBC == MBC_MBC3) {
      if (s.rtc_sub + (cyc & s.rtc_run) >= RTC_CPS) s.rtc_tick(cyc);
      else s.rtc_sub += cyc & s.rtc_run;
    }
    cyc_total += cyc;
    cycle_frame += cyc;
    if (cycle_frame >= CYCLES_PER_FRAME) {
      do {
        cycle_frame -= CYCLES_PER_FRAME;
        s.frames_done++;
      } while (cycle_frame >= CYCLES_PER_FRAME && s.frames_done < frames_to_run);
    }
  }
  s.materialize();

  // ---- post-step body (post_step.py:11-102) ----
  const int a = s.A(), b = s.getr(0), c = s.getr(1), d = s.getr(2);
  const int e_ = s.getr(3), h = s.getr(4), l = s.getr(5);
  if (stage == STAGE_OBS || stage == STAGE_FULL) {
    float* o = st.obs + (size_t)env * OBS_DIM;
    int m[16];
#pragma unroll
    for (int k = 0; k < 16; k++) m[k] = s.M(0xC000 + k);
    float4 q[8];
    q[0] = make_float4((float)(s.pc & 0xFFFF) / 65535.0f, (float)(s.sp & 0xFFFF) / 65535.0f,
                       (float)a / 255.0f, (float)(s.f & 0xFF) / 255.0f);
    q[1] = make_float4((float)b / 255.0f, (float)c / 255.0f, (float)d / 255.0f, (float)e_ / 255.0f);
    q[2] = make_float4((float)h / 255.0f, (float)l / 255.0f, (float)m[0] / 255.0f, (float)m[1] / 255.0f);
    q[3] = make_float4((float)m[2] / 255.0f, (float)m[3] / 255.0f, (float)m[4] / 255.0f, (float)m[5] / 255.0f);
    q[4] = make_float4((float)m[6] / 255.0f, (float)m[7] / 255.0f, (float)m[8] / 255.0f, (float)m[9] / 255.0f);
    q[5] = make_float4((float)m[10] / 255.0f, (float)m[11] / 255.0f, (float)m[12] / 255.0f, (float)m[13] / 255.0f);
    q[6] = make_float4((float)m[14] / 255.0f, (float)m[15] / 255.0f, (float)((m[0] ^ m[1]) & 0xFF) / 255.0f,
                       (float)((m[2] + m[3] * 5) & 0xFF) / 255.0f);
    q[7] = make_float4((float)((m[4] ^ a) & 0xFF) / 255.0f, (float)((m[5] + b) & 0xFF) / 255.0f,
                       (float)((m[6] ^ c) & 0xFF) / 255.0f, (float)((m[7] + d) & 0xFF) / 255.0f);
    float4* o4 = reinterpret_cast<float4*>(o);
#pragma unroll
    for (int k = 0; k < 8; k++) o4[k] = q[k];
  }
  if (stage == STAGE_REWARD || stage == STAGE_FULL) {
    int mix = (s.M(0xC000) + s.M(0xC001) * 3) & 0xFF;
    st.reward[env] = (float)((a ^ mix) & 0xFF) / 255.0f;
  }

  // ---- write-back ----
  int32_t* O = st.i32 + env;
  auto stv = [&](int fld, int v) { O[(size_t)fld * S] = v; };
  stv(F_PC, s.pc & 0xFFFF); stv(F_SP, s.sp & 0xFFFF);
  stv(F_A, a); stv(F_B, b); stv(F_C, c); stv(F_D, d); stv(F_E, e_); stv(F_H, h); stv(F_L, l);
  stv(F_F, s.f & 0xF0);
  stv(F_CYCLE_IN_FRAME, cycle_frame);
  stv(F_TRAP_FLAG, s.trap);
  stv(F_IME, s.ime); stv(F_IME_DELAY, s.ime_delay); stv(F_HALTED, s.halted);
  stv(F_DIV_COUNTER, s.div); stv(F_TIMER_PREV_IN, s.prev_in);
  stv(F_TIMA_RELOAD_PENDING, s.rl_pending); stv(F_TIMA_RELOAD_DELAY, s.rl_delay);
  stv(F_PPU_SCANLINE_CYCLE, s.scan); stv(F_PPU_LY, s.ly); stv(F_PPU_WINDOW_LINE, s.wl);
  st.u8s[(size_t)F_STAT_PREV * S + env] = (uint8_t)s.stat_prev;
  st.i64[(size_t)F_INSTR_COUNT * S + env] = instr;
  st.i64[(size_t)F_CYCLE_COUNT * S + env] = cyc_total;
  s.M(0xFF00) = (uint8_t)s.joyp; s.M(0xFF04) = (uint8_t)s.div_b; s.M(0xFF05) = (uint8_t)s.tima;
  s.M(0xFF06) = (uint8_t)s.tma; s.M(0xFF07) = (uint8_t)s.tac; s.M(0xFF0F) = (uint8_t)s.iflag;
  s.M(0xFF40) = (uint8_t)s.lcdc; s.M(0xFF41) = (uint8_t)s.stat; s.M(0xFF44) = (uint8_t)s.ly_b;
  s.M(0xFF45) = (uint8_t)s.lyc; s.M(0xFF4A) = (uint8_t)s.wy; s.M(0xFFFF) = (uint8_t)s.ie;
  int32_t* CW = st.cart_state + env;
  CW[(size_t)CS_RAM_ENABLE * S] = s.ram_en;
  CW[(size_t)CS_ROM_BANK_LO * S] = s.bank_lo;
  CW[(size_t)CS_ROM_BANK_HI * S] = s.bank_hi;
  CW[(size_t)CS_RAM_BANK * S] = s.ram_bank;
  CW[(size_t)CS_BANK_MODE * S] = s.bank_mode;
  CW[(size_t)CS_BOOTROM * S] = s.bootrom;
  CW[(size_t)CS_RTC_SELECT * S] = s.rtc_sel;
  CW[(size_t)CS_RTC_LATCH * S] = s.rtc_latch;
  if (MBC == MBC_MBC3) {
    CW[(size_t)CS_RTC_S * S] = s.rtc_s;
    CW[(size_t)CS_RTC_M * S] = s.rtc_m;
    CW[(size_t)CS_RTC_H * S] = s.rtc_h;
    CW[(size_t)CS_RTC_DL * S] = s.rtc_dl;
    CW[(size_t)CS_RTC_DH * S] = s.rtc_dh;
    CW[(size_t)CS_RTC_LAST * S] = s.rtc_sub;
  }
}

// ---------------------------------------------------------------------------
// Host launcher
// ---------------------------------------------------------------------------
size_t step_smem_bytes(const DevState& st) {
  int r = st.rom_bytes < ROM_SMEM_MAX ? st.rom_bytes : ROM_SMEM_MAX;
  return 768 + (size_t)((r + 15) & ~15);
}

static int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return v && *v ? atoi(v) : dflt;
}

// Envs per warp and register cap for a batch of n envs (overridable with
// GBX_ENVS_PER_WARP / GBX_STEP_REGCAP for measurements).
void step_launch_shape(int n, int* K, int* regcap) {
  int k = env_int("GBX_ENVS_PER_WARP", 0);
  int rc = env_int("GBX_STEP_REGCAP", -1);
  if (k <= 0) k = 32;
  if (k > 32) k = 32;
  *K = k;
  *regcap = rc < 0 ? 0 : (rc ? 1 : 0);
}

template <int MBC>
static cudaError_t launch_mbc(const DevState& st, const int32_t* actions, int frames, int release, int stage,
                              cudaStream_t stream, int K, int regcap, size_t sm) {
  const int threads = 256;
  const long long warps = (st.n + K - 1) / K;
  const int blocks = (int)((warps * 32 + threads - 1) / threads);
  if (regcap) {
    cudaFuncSetAttribute(gb_step_kernel<MBC, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    gb_step_kernel<MBC, 1><<<blocks, threads, sm, stream>>>(st, actions, frames, release, stage, K);
  } else {
    cudaFuncSetAttribute(gb_step_kernel<MBC, 0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    gb_step_kernel<MBC, 0><<<blocks, threads, sm, stream>>>(st, actions, frames, release, stage, K);
  }
  return cudaGetLastError();
}

cudaError_t launch_step(const DevState& st, const int32_t* actions, int frames, int release, int stage,
                        cudaStream_t stream) {
  const size_t sm = step_smem_bytes(st);
  int K, regcap;
  step_launch_shape(st.n, &K, &regcap);
  switch (st.mbc_kind) {
    case MBC_MBC1: return launch_mbc<MBC_MBC1>(st, actions, frames, release, stage, stream, K, regcap, sm);
    case MBC_MBC3: return launch_mbc<MBC_MBC3>(st, actions, frames, release, stage, stream, K, regcap, sm);
    default: return launch_mbc<MBC_ROM_ONLY>(st, actions, frames, release, stage, stream, K, regcap, sm);
  }
}

}  // namespace gbx
