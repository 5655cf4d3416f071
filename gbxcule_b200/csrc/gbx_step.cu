// gbx_step.cu - the env-step kernel: one SM83 console per thread for the whole
// frame-skip loop, with two interpreters: a switch over instruction families
// (below) and a uniform datapath for full warps of envs at different PCs
// (uniform_loop, gbx_udesc.h). The host picks K envs per warp and the
// interpreter per batch by timing (gbx_api.cu).
//
// Semantics follow the reference kernel of bkase/gbxcule
// (src/gbxcule/kernels/cpu_step_builder.py:876-1781 and the instruction
// templates in src/gbxcule/kernels/cpu_templates/), quirks included. The
// structure does not: the reference re-reads and re-writes per-env arrays in
// global memory for every register, IO port and timer field on every
// instruction; here that state lives in registers for the whole launch and
// goes back to HBM once at the end.
//
//  * Memory: env-major (gbx_layout.h): each env's stack, HRAM and IO page sit
//    in cache lines of their own, so envs on different warps never write the
//    same sector. Cached IO ports (JOYP, DIV, TIMA, TMA, TAC, IF, LCDC, STAT, LY,
//    LYC, WY, IE) live in registers; every path that touches those addresses
//    (CPU access, OAM DMA source, env-0 latches) goes through the cache.
//  * Fetch (switch): the ROM is pre-decoded on the host into one 32-bit word
//    per byte (opcode, 16-bit immediate, family). Banks 0-1 of it sit in
//    shared memory, so fetch + decode is a single 4-byte shared load; other
//    banks come through the read-only path. (Uniform: raw ROM bytes, two
//    aligned words per fetch.) Code outside ROM (RAM, the boot ROM overlay,
//    bank-crossing fetches) is decoded from bytes.
//  * Execute (switch): one switch over 36 families of SM83's regular encoding (the
//    CB and ALU register forms split by operation). Registers are packed
//    into two u32, read with one byte-permute and written with one bit-field
//    insert; operand fields are extracted inside the cases that use them;
//    memory operands are read inside their families (plain RAM, the mapped
//    cart-RAM bank and JOYP inline, the rest out of line); one write site.
//  * Post-instruction work is lazy. The reference updates timer, DIV, STAT
//    mode bits, stat_prev, LY, RTC and the frame counter after every
//    instruction. Here one counter `clk` accumulates cycles and is compared
//    with `next_ev`, the cycles until the earliest event (timer edge/reload,
//    scanline boundary, frame end, RTC second). Until then every one of those
//    values is a function of the state at the last sync plus `clk`, so the
//    common instruction tail is `clk += cyc; if (clk >= next_ev) ...`. An
//    instruction that crosses an event, halts, traps, writes a port with
//    timing side effects (LCDC, STAT, LY, LYC, WY, IF, IE, timer, RTC) or
//    sets IME from 0 forces `next_ev` and runs the reference's
//    post-processing verbatim on materialised state (slow_post). The
//    reference's timer_tick is additive over time, so lumping event-free
//    cycles is exact.
//  * HALT: runs of 4-cycle halted iterations that cannot change anything
//    observable except counters (no line boundary, no timer reload, no frame
//    end) are applied in one batch.
#include <cuda_runtime.h>
#include <limits.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "gbx_layout.h"
#include "gbx_udesc.h"

namespace gbx {

// ---------------------------------------------------------------------------
// Decode
// ---------------------------------------------------------------------------
enum Family : uint8_t {
  FM_LDRR, FM_LD16, FM_ST_A, FM_LD_A, FM_INCDEC16, FM_INCDEC8, FM_INCDEC_HL, FM_LD8_IMM,
  FM_ST_HL_IMM, FM_ROTA, FM_ST_SP16, FM_ADDHL, FM_TRAP, FM_JR, FM_DAA, FM_FLAGOP,
  FM_LDR_HL, FM_STHL_R, FM_HALT, FM_ALU_V, FM_RET, FM_POP, FM_JP,
  FM_CALL, FM_PUSH, FM_RST, FM_CB_HL, FM_SPADD, FM_IME,
  // register-operand forms split by operation, so their cases hold no inner dispatch
  FM_CB_ROT, FM_CB_BIT, FM_CB_RES, FM_CB_SET, FM_ALU_ADC, FM_ALU_SBC, FM_ALU_LOG
};

// CB-prefixed instructions take their family from the second byte
__host__ __device__ constexpr uint8_t cb_family(int b1) {
  return (b1 & 7) == 6 ? FM_CB_HL : (uint8_t)(FM_CB_ROT + (b1 >> 6));
}

// family of an unprefixed opcode (0xCB: see cb_family)
__host__ __device__ constexpr uint8_t decode_entry(int op) {
  int x = op >> 6, y = (op >> 3) & 7, z = op & 7;
  if (op == 0xCB) return FM_CB_HL;
  if (op == 0x10 || op == 0xD3 || op == 0xDB || op == 0xDD || op == 0xE3 || op == 0xE4 ||
      op == 0xEB || op == 0xEC || op == 0xED || op == 0xF4 || op == 0xFC || op == 0xFD)
    return FM_TRAP;
  if (x == 1) {
    if (op == 0x76) return FM_HALT;
    if (z == 6) return FM_LDR_HL;
    if (y == 6) return FM_STHL_R;
    return FM_LDRR;
  }
  if (x == 2) return z == 6 ? FM_ALU_V : y < 2 ? FM_ALU_ADC : (y < 4 || y == 7) ? FM_ALU_SBC : FM_ALU_LOG;
  if (x == 0) {
    switch (z) {
      case 0: return op == 0x00 ? FM_LDRR : op == 0x08 ? FM_ST_SP16 : FM_JR;
      case 1: return (y & 1) ? FM_ADDHL : FM_LD16;
      case 2:
        if (y & 1) return FM_LD_A;
        return FM_ST_A;
      case 3: return FM_INCDEC16;
      case 4: case 5: return y == 6 ? FM_INCDEC_HL : FM_INCDEC8;
      case 6: return y == 6 ? FM_ST_HL_IMM : FM_LD8_IMM;
      default: return y == 4 ? FM_DAA : y >= 5 ? FM_FLAGOP : FM_ROTA;
    }
  }
  switch (op) {  // x == 3
    case 0xC0: case 0xC8: case 0xD0: case 0xD8: case 0xC9: case 0xD9:
      return FM_RET;
    case 0xC1: case 0xD1: case 0xE1: case 0xF1: return FM_POP;
    case 0xC2: case 0xCA: case 0xD2: case 0xDA: case 0xC3: case 0xE9: return FM_JP;
    case 0xC4: case 0xCC: case 0xD4: case 0xDC: case 0xCD: return FM_CALL;
    case 0xC5: case 0xD5: case 0xE5: case 0xF5: return FM_PUSH;
    case 0xE0: case 0xE2: case 0xEA: return FM_ST_A;
    case 0xF0: case 0xF2: case 0xFA: return FM_LD_A;
    case 0xE8: case 0xF8: case 0xF9: return FM_SPADD;
    case 0xF3: case 0xFB: return FM_IME;
    default: break;
  }
  if (z == 6) return FM_ALU_V;  // ALU A,d8
  return FM_RST;                // z == 7
}

// 32-bit decoded instruction: opcode | imm16 << 8 | entry << 24
__host__ __device__ constexpr uint32_t decode_word(int op, int b1, int b2) {
  const uint32_t e = op == 0xCB ? cb_family(b1) : decode_entry(op);
  return (uint32_t)op | ((uint32_t)b1 << 8) | ((uint32_t)b2 << 16) | (e << 24);
}

struct DecodeTable {
  uint8_t e[256];
};
__host__ __device__ constexpr DecodeTable make_table() {
  DecodeTable t{};
  for (int i = 0; i < 256; i++) t.e[i] = decode_entry(i);
  return t;
}
__constant__ DecodeTable c_decode = make_table();
// descriptors and rotate table of the uniform interpreter (gbx_udesc.h),
// staged in shared memory
__constant__ UDescTable c_udesc = make_udesc_table();
__constant__ RotTable c_rot = make_rot_table();

// Host: pre-decode a ROM image (every byte offset as an instruction start).
void predecode_rom(const uint8_t* rom, int n, uint32_t* out) {
  for (int i = 0; i < n; i++) {
    int b1 = i + 1 < n ? rom[i + 1] : 0, b2 = i + 2 < n ? rom[i + 2] : 0;
    out[i] = decode_word(rom[i], b1, b2);
  }
}

// ---------------------------------------------------------------------------
// Per-thread emulator state
// ---------------------------------------------------------------------------
#define FLAGS(z, n, h, c) ((((z) ? 1 : 0) << 7) | (((n) ? 1 : 0) << 6) | (((h) ? 1 : 0) << 5) | (((c) ? 1 : 0) << 4))

// events that send an instruction's post-processing down the exact path
enum Event { EV_FIRST = 1, EV_HALT = 2, EV_TRAP = 4, EV_LCDC = 8, EV_PPU = 16, EV_RTC = 32, EV_IRQ = 64,
             EV_TIMER = 128 };

// CPU registers and the event clock: the only state the interpreter loop
// keeps in registers. Everything else lives in Emu, in local memory, and is
// touched by the out-of-line slow paths only.
// RLC RRC RL RR SLA SRA SWAP SRL of v (bitops.py); oc = carry in, c = carry out
__device__ __forceinline__ int cb_rot(int kind, int v, int oc, int& c) {
  switch (kind) {
    case 0: c = v >> 7; return ((v << 1) & 0xFF) | c;
    case 1: c = v & 1; return (v >> 1) | (c << 7);
    case 2: c = v >> 7; return ((v << 1) & 0xFF) | oc;
    case 3: c = v & 1; return (v >> 1) | (oc << 7);
    case 4: c = v >> 7; return (v << 1) & 0xFF;
    case 5: c = v & 1; return (v >> 1) | (v & 0x80);
    case 6: c = 0; return ((v & 0xF) << 4) | (v >> 4);
    default: c = v & 1; return v >> 1;
  }
}

struct Hot {
  uint32_t bcde, hlxa;  // B C D E | H L - A, high byte first
  int f, pc, sp;
  int clk, next_ev;     // cycles since the last sync; cycles to the next event

  __device__ __forceinline__ int A() const { return hlxa & 0xFF; }
  __device__ __forceinline__ void setA(int v) { hlxa = (hlxa & 0xFFFFFF00u) | (uint32_t)(v & 0xFF); }
  __device__ __forceinline__ int HL() const { return hlxa >> 16; }
  __device__ __forceinline__ void setHL(int v) { hlxa = (hlxa & 0xFFFFu) | ((uint32_t)(v & 0xFFFF) << 16); }
  __device__ __forceinline__ int BC() const { return bcde >> 16; }
  __device__ __forceinline__ int DE() const { return bcde & 0xFFFF; }
  __device__ __forceinline__ int C_() const { return (bcde >> 16) & 0xFF; }
  // r8 index 0..7: 0 B, 1 C, 2 D, 3 E, 4 H, 5 L, 7 A (6 = (HL), never passed;
  // the decode sends every (HL) form to its own family). {bcde, hlxa} read
  // as one 8-byte array puts register i at byte i ^ 3; byte 5 (hlxa's unused
  // byte) is always 0, so selecting it for the upper three result bytes
  // returns the register zero-extended without a mask.
  __device__ __forceinline__ int getr(int i) const {
    return __byte_perm(bcde, hlxa, (i ^ 3) | 0x5550);
  }
  __device__ __forceinline__ static uint32_t insert_byte(uint32_t w, int v, int pos) {
    uint32_t r;
    asm("bfi.b32 %0, %1, %2, %3, 8;" : "=r"(r) : "r"(v), "r"(w), "r"(pos));
    return r;
  }
  __device__ __forceinline__ void setr(int i, int v) {  // v: low 8 bits are stored
    const int pos = (~i & 3) << 3;
    if (i & 4) hlxa = insert_byte(hlxa, v, pos); else bcde = insert_byte(bcde, v, pos);
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
  // ALU kinds ADD ADC SUB SBC AND XOR OR CP (alu.py)
  __device__ __forceinline__ void alu(int kind, int v) {
    const int a = A();
    int r;
    switch (kind) {
      case 0: case 1: {
        const int cin = kind == 1 ? (f >> 4) & 1 : 0;
        r = a + v + cin;
        f = (((r & 0xFF) == 0) << 7) | ((((a & 0xF) + (v & 0xF) + cin) > 0xF) << 5) | ((r > 0xFF) << 4);
        setA(r);
        return;
      }
      case 2: case 3: case 7: {
        const int cin = kind == 3 ? (f >> 4) & 1 : 0;
        r = a - v - cin;
        f = (((r & 0xFF) == 0) << 7) | 0x40 | ((((a & 0xF) - (v & 0xF) - cin) < 0) << 5) | ((r < 0) << 4);
        if (kind != 7) setA(r);
        return;
      }
      case 4: r = a & v; f = ((r == 0) << 7) | 0x20; break;
      case 5: r = a ^ v; f = (r == 0) << 7; break;
      default: r = a | v; f = (r == 0) << 7; break;
    }
    setA(r);
  }
  // DAA (alu.py)
  __device__ __forceinline__ void daa() {
    int a = A(), n = (f >> 6) & 1, hf = (f >> 5) & 1, c = (f >> 4) & 1, adj = 0, carry = c;
    if (!n) {
      if (hf || (a & 0xF) > 9) adj |= 0x06;
      if (c || a > 0x99) { adj |= 0x60; carry = 1; }
      a = (a + adj) & 0xFF;
    } else {
      if (hf) adj |= 0x06;
      if (c) adj |= 0x60;
      a = (a - adj) & 0xFF;
    }
    f = FLAGS(a == 0, n, 0, carry);
    setA(a);
  }
  __device__ __forceinline__ bool cond(int cc) const {
    int bit = (cc & 2) ? ((f >> 4) & 1) : ((f >> 7) & 1);
    return (cc & 1) ? bit : !bit;
  }
};

template <int MBC>
struct Emu {
  // addressing
  uint8_t* mem;           // env's 64 KiB address space (env-major)
  uint32_t S;             // SoA row stride of the scalar fields
  const uint32_t* pre_s;  // shared memory: pre-decoded rom[0 .. pre_s_words)
  const uint32_t* pre_g;  // global pre-decoded ROM
  const uint8_t* boot_s;  // shared memory: boot ROM
  const uint8_t* rom_g;   // global ROM bytes
  int32_t* cart_state;    // &st.cart_state[env]
  uint8_t* cart_ram;      // env's cartridge RAM (env-major)
  uint8_t* serial;        // env's serial capture buffer (env-major)
  int32_t* i32;           // &st.i32[env]
  uint8_t* u8s;           // &st.u8s[env]
  uint8_t* latch;         // st.latch
  int rom_bank_count, rom_bank_mask, ram_bank_count;
  int pre_s_words;
  int is_env0;
  // CPU (the interpreter loop's registers, copied in around slow paths)
  uint32_t bcde, hlxa;   // B C D E | H L - A, high byte first
  int f, pc, sp;
  int ime, ime_delay, halted;
  int trap;
  // cached IO ports (values of mem[FFxx]); stat/div_b/prev_in/stat_prev are
  // exact only while lazy == 0
  int joyp, div_b, tima, tma, tac, iflag, lcdc, stat, ly_b, lyc, wy, ie;
  // timer
  int div, rl_pending, rl_delay, prev_in;
  // PPU
  int scan, ly, wl, stat_prev;
  // cart
  int ram_en, bank_lo, bank_hi, ram_bank, bank_mode, bootrom, rtc_sel, rtc_latch;
  int bank0_off, bankN_off;   // ROM byte offset of a bank region; -1 when out of range
  int win_hi;                 // fetch window: pc in [0, win_hi) reads pre_s[pc]
  int cram_off;               // cart RAM offset of the bank at A000-BFFF; -1 when such
                              // accesses need the full path (disabled, absent, RTC)
  int rtc_sub, rtc_s, rtc_m, rtc_h, rtc_dl, rtc_dh;
  // step
  int frames_done, release, action;
  int cycle_frame, cyc_run, ninstr;
  // lazy state
  int lazy, ev, clk, next_ev, stat_hi, lcd_on, rtc_run, lcdc_before;

  // ---- memory -------------------------------------------------------------
  __device__ __forceinline__ uint8_t& M(int a) const { return mem[a]; }

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
    // Shared memory holds the pre-decoded words of ROM offsets [0, pre_s_words).
    // With bank 0 at offset 0 the bank-0 region fetches from it (minus the
    // boot ROM overlay and the last two bytes, whose instruction could reach
    // into bank N); with bank 1 also mapped the window spans both regions.
    // While the boot ROM overlays 0000-00FF the window is empty (a boot ROM
    // runs inside its overlay, which the full fetch path serves anyway), so
    // the window test is one unsigned compare.
    int hi = 0;
    if (!bootrom && bank0_off == 0) hi = (bankN_off == 0 && pre_s_words >= 0x8000) ? 0x7FFE : 0x3FFE;
    if (hi > pre_s_words) hi = pre_s_words;  // only the staged words are in shared memory
    win_hi = hi;
    // A000-BFFF as plain bytes when it maps a whole bank of cart RAM
    // (ram_index / cart_read with RAM enabled and no RTC register selected)
    cram_off = -1;
    if (ram_bank_count > 0 && ram_en != 0) {
      const int sel = rtc_sel & 0x0F;
      if (!(MBC == MBC_MBC3 && sel >= 0x08 && sel <= 0x0C)) {
        int rb = 0;
        if (MBC == MBC_MBC1) { if (bank_mode & 1) rb = ram_bank & 3; }
        else if (MBC == MBC_MBC3) rb = ram_bank & 3;
        cram_off = (rb % ram_bank_count) * RAM_BANK;
      }
    }
  }

  __device__ __forceinline__ int rom_read(int a) const {
    if (a < 0x100 && bootrom) return boot_s[a];
    int off = a < 0x4000 ? bank0_off : bankN_off;
    if (off < 0) return 0xFF;
    return __ldg(rom_g + off + a);
  }

  // STAT low bits / stat_prev / LY / DIV / TIMA as functions of the state at
  // the last sync plus clk (lazy mode). A lazy period may cross scanlines
  // (never VBlank entry or the wrap to line 0) and TIMA edges (never an
  // overflow), see delazify().
  __device__ __forceinline__ static int mode_at(int line, int sc) {
    return line >= SCREEN_H ? 1 : sc < 80 ? 2 : sc < 250 ? 3 : 0;
  }
  __device__ __forceinline__ int ppu_mode_at(int sc) const { return mode_at(ly, sc); }
  __device__ __forceinline__ static int prev_bits(int mode, int coinc) {
    return (mode == 0) | ((mode == 1) << 1) | ((mode == 2) << 2) | (coinc << 3);
  }
  __device__ __forceinline__ int stat_now() const {
    if (!lazy) return stat;
    if (!lcd_on) return stat_hi | ((ly == lyc) << 2);
    const int t = scan + clk, n = t / CYCLES_PER_LINE, line = ly + n;
    return stat_hi | ((line == lyc) << 2) | mode_at(line, t - n * CYCLES_PER_LINE);
  }
  __device__ __forceinline__ int ly_b_now() const {
    if (!lazy || !lcd_on) return ly_b;
    const int n = (scan + clk) / CYCLES_PER_LINE;
    return n ? ly + n : ly_b;
  }
  __device__ __forceinline__ int div_byte_now() const {
    return lazy ? (((div + clk) >> 8) & 0xFF) : div_b;
  }
  __device__ __forceinline__ int tima_now() const {
    if (!lazy || !(tac & 4) || rl_pending) return tima;
    const int sh = div_bit(tac) + 1;
    return tima + (((div & ((1 << sh) - 1)) + clk) >> sh);
  }

  __device__ __forceinline__ int io_read(int a) const {
    switch (a & 0xFF) {
      case 0x00: return joyp;
      case 0x04: return div_byte_now();
      case 0x05: return tima_now();
      case 0x06: return tma;
      case 0x07: return tac;
      case 0x0F: return iflag;
      case 0x40: return lcdc;
      case 0x41: return stat_now();
      case 0x44: return ly_b_now();
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
    return cart_ram[off];
  }

  // read8 (:539-657); region = a >> 13: 4 VRAM and 6 WRAM first
  __device__ __forceinline__ int read8(int addr) const {
    const int a = addr & 0xFFFF;
    const int r = a >> 13;
    if ((r | 2) == 6) return M(a);
    if (r < 4) return rom_read(a);
    if (r == 5) return cart_read(a);
    if (a >= 0xFF00) return io_read(a);
    return M(a < 0xFE00 ? a - 0x2000 : a);
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
  // the reference's timer_tick, exact. Without a pending reload and with no
  // overflow inside `cycles`, its edge loop only counts TIMA edges, which is
  // done in closed form.
  __device__ void timer_tick(int cycles) {
    if (cycles <= 0) return;
    int edges = 0;
    if (!rl_pending && (tac & 4)) {
      const int sh = div_bit(tac) + 1;
      edges = ((div & ((1 << sh) - 1)) + cycles) >> sh;
    }
    if (!rl_pending && tima + edges <= 0xFF) {
      div = (div + cycles) & 0xFFFF;
      tima += edges;
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
  // cycles from now until timer_tick does more than advance DIV and count
  // TIMA edges: the overflow edge, or while a reload is pending the reload
  // and the next edge
  __device__ __forceinline__ int timer_event() const {
    int t = INT_MAX;
    if (rl_pending) t = rl_delay;
    if (tac & 4) {
      int period = 1 << (div_bit(tac) + 1);
      int e = period - (div & (period - 1));
      if (!rl_pending) e += (0xFF - tima) * period;
      t = e < t ? e : t;
    }
    return t;
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
    while (lines > 0) {
      int prev = ly;
      if (prev < SCREEN_H && (l & 0x20) && prev >= wy) wl++;
      ly = ly + 1 == LINES_PER_FRAME ? 0 : ly + 1;
      if (ly == 0) wl = 0;
      ly_b = ly;
      // ppu_update_stat_irq: rising edge of an enabled condition sets IF bit 1
      int keep = stat & 0xF8, c = ly == lyc, mode = ly >= SCREEN_H ? 1 : 0;
      stat = keep | (c << 2) | mode;
      int cur = prev_bits(mode, c);
      if ((keep >> 3) & cur & ~(stat_prev & 0xF)) iflag |= 0x02;
      stat_prev = cur;
      if (prev == 143 && ly == 144) iflag |= 0x01;
      if (ly < SCREEN_H) latch0(ly);
      lines--;
    }
    int mode = ppu_mode_at(scan);
    int c = ly == lyc;
    stat = (stat & 0xF8) | (c << 2) | mode;
    stat_prev = prev_bits(mode, c);
    return l;
  }

  // ---- lazy <-> exact --------------------------------------------------------
  // Advance every lazily tracked counter by q event-free cycles.
  __device__ void apply_quiet(int q) {
    if (q <= 0) return;
    timer_tick(q);  // no overflow or reload inside q (q < next_ev)
    if (lcd_on) {
      // whole scanlines inside q: none of them enters VBlank or wraps, and
      // with the STAT interrupt enables clear each one only moves LY, LY's
      // register and the window line (ppu_advance's per-line body)
      const int t = scan + q;
      if (t >= CYCLES_PER_LINE) {
        const int n = t / CYCLES_PER_LINE;
        scan = t - n * CYCLES_PER_LINE;
        if (lcdc & 0x20) {
          const int lo = ly > wy ? ly : wy, hi = ly + n < SCREEN_H ? ly + n : SCREEN_H;
          if (hi > lo) wl += hi - lo;
        }
        ly += n;
        ly_b = ly;
      } else {
        scan = t;
      }
    }
    if (MBC == MBC_MBC3) rtc_sub += q & rtc_run;
    cycle_frame += q;
    cyc_run += q;
  }
  // Turn derived values into stored ones (clk must be 0).
  __device__ void materialize() {
    if (!lazy) return;
    stat = stat_hi | ((ly == lyc) << 2) | (lcd_on ? ppu_mode_at(scan) : 0);
    stat_prev = lcd_on ? prev_bits(ppu_mode_at(scan), ly == lyc) : 0;
    div_b = (div >> 8) & 0xFF;
    prev_in = timer_in(div, tac);
    lazy = 0;
  }
  // Bring everything up to date (apply clk, materialise).
  __device__ void sync_all() {
    if (!lazy) return;
    apply_quiet(clk);
    clk = 0;
    materialize();
  }
  // After exact processing: derived values agree with the state again.
  __device__ void delazify() {
    lazy = 1;
    stat_hi = stat & 0xF8;
    lcd_on = (lcdc & 0x80) != 0;
    rtc_run = (MBC == MBC_MBC3 && !(rtc_dh & 0x40) && rtc_sub >= 0) ? -1 : 0;
    int t = timer_event();
    if (lcd_on) {
      int p = CYCLES_PER_LINE - scan;  // next scanline
      // Line changes only need the exact path when they can raise a STAT
      // interrupt, enter VBlank, wrap to line 0 or latch env 0's registers.
      if (!is_env0 && !(stat_hi & 0x78))
        p += ((ly < SCREEN_H ? SCREEN_H : LINES_PER_FRAME) - 1 - ly) * CYCLES_PER_LINE;
      t = p < t ? p : t;
    }
    { int fr = CYCLES_PER_FRAME - cycle_frame; t = fr < t ? fr : t; }
    if (MBC == MBC_MBC3 && rtc_run) { int r = RTC_CPS - rtc_sub; t = r < t ? r : t; }
    next_ev = t;
    clk = 0;
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

  // JOYP's value for select bits 00, 10, 20, 30 (bytes 0..3); changes only
  // when frames_done crosses the release frame
  __device__ __forceinline__ uint32_t joyp_table() const {
    return (uint32_t)joyp_value(0x00) | ((uint32_t)joyp_value(0x10) << 8) | ((uint32_t)joyp_value(0x20) << 16) |
           ((uint32_t)joyp_value(0x30) << 24);
  }
  // JOYP select write: the register latches the selected group's buttons
  __device__ __forceinline__ void write_joyp(int val) {
    const int sel = val & 0x30;
    u8s[(size_t)F_JOYP_SELECT * S] = (uint8_t)sel;
    joyp = joyp_value(sel);
  }

  __device__ void write_io(int a, int val) {
    const int v8 = val & 0xFF;
    switch (a & 0xFF) {
      case 0x00: write_joyp(v8); return;
      case 0x0F: iflag = v8 & 0x1F; ev |= EV_IRQ; return;
      case 0x02:
        if ((val & 0x80) && (val & 0x01)) {
          int idx = i32[(size_t)F_SERIAL_LEN * S];
          if (idx < SERIAL_MAX) {
            serial[idx] = M(0xFF01);
            i32[(size_t)F_SERIAL_LEN * S] = idx + 1;
          } else {
            u8s[(size_t)F_SERIAL_OVERFLOW * S] = 1;
          }
          M(0xFF02) = (uint8_t)(val & 0x7F);
          iflag |= 0x08;
          ev |= EV_IRQ;
        } else {
          M(0xFF02) = (uint8_t)v8;
        }
        return;
      case 0x50:
        if (val != 0) { bootrom = 0; update_banks(); }
        return;
      case 0x04: case 0x05: case 0x06: case 0x07: {
        sync_all();
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
        ev |= EV_TIMER;
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
      case 0xFF: ie = v8 & 0x1F; ev |= EV_IRQ; return;
      case 0x40:
        sync_all();  // lines so far ran under the old LCDC
        if (!(ev & EV_LCDC)) lcdc_before = lcdc;
        lcdc = v8;
        ev |= EV_LCDC;
        return;
      case 0x41:
        sync_all();  // interrupt enables change which line changes matter
        stat = v8; stat_hi = v8 & 0xF8;
        ev |= EV_PPU;
        return;
      case 0x44: sync_all(); ly_b = v8; ev |= EV_PPU; return;
      case 0x45:
        // stat_prev of the last refresh was computed with the old LYC
        sync_all();
        lyc = v8;
        ev |= EV_PPU;
        return;
      case 0x4A: sync_all(); wy = v8; ev |= EV_PPU; return;  // the window line count uses WY
      default: M(a) = (uint8_t)v8; return;
    }
  }

  __device__ void write8_slow(int a, int val) {
    const int v8 = val & 0xFF;
    if (a >= 0xFF00) { write_io(a, val); return; }
    if (a >= 0xE000 && a < 0xFE00) { M(a - 0x2000) = (uint8_t)v8; return; }
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
      if (off >= 0) cart_ram[off] = (uint8_t)v8;
      return;
    }
    if (a < 0x8000) { write_mbc(a, val); return; }
    M(a) = (uint8_t)v8;  // FE00-FEFF
  }

  // cartridge register write (0000-7FFF): RAM enable, bank selects, RTC latch
  __device__ __forceinline__ void write_mbc(int a, int val) {
    {
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
        update_banks();
      }
    }
  }

  __device__ __forceinline__ void write8(int addr, int val) {
    const int a = addr & 0xFFFF;
    if (((a >> 13) | 2) == 6) { M(a) = (uint8_t)val; return; }  // VRAM, WRAM
    write8_slow(a, val);
  }

  // interrupt service (:1502-1604): IME off, IF bit cleared, PC pushed
  __device__ void service(int pending) {
    int bit = pending & (-pending);  // lowest set bit = highest priority
    int vector = 0x40 + 8 * (31 - __clz(bit));
    ime = 0;
    iflag &= 0xFF ^ bit;
    int ret = pc;
    sp = (sp - 1) & 0xFFFF;
    write8(sp, ret >> 8);
    sp = (sp - 1) & 0xFFFF;
    write8(sp, ret & 0xFF);
    pc = vector;
  }

  // ---- exact per-instruction tail (:1375-1758) ---------------------------------
  // Runs after an instruction of `cyc` cycles whose tail could not stay lazy.
  __device__ void slow_post(int cyc, int opcode, int pc_before, int frames_to_run) {
    const int lcdc_prev = ((ev & EV_LCDC) ? lcdc_before : lcdc) & 0x80;
    if (lazy) {
      apply_quiet(clk - cyc);  // the event-free cycles of earlier instructions
      clk = 0;
      materialize();
    }
    timer_tick(cyc);
    if (ime_delay) { ime = 1; ime_delay = 0; }
    int lcdc_now = ppu_advance(cyc);
    const int pending = ie & iflag & 0x1F;
    int svc = 0;
    if (pending) {
      if (halted) halted = 0;
      if (ime) {
        service(pending);
        svc = 20;
        timer_tick(20);
        lcdc_now = ppu_advance(20);
      }
    }
    const int total = cyc + svc;
    rtc_tick(total);
    cyc_run += total;
    cycle_frame += total;
    if (lcdc_prev && !(lcdc_now & 0x80)) {
      int tail = total;
      if (opcode == 0xE0 && (read8((pc_before + 1) & 0xFFFF) & 0xFF) == 0x40 && cyc >= 4) tail = total - 4;
      cycle_frame = tail;
      frames_done++;
    } else if (!lcdc_prev && (lcdc_now & 0x80)) {
      scan = 0; ly = 0; wl = 0; ly_b = 0;
      stat = (stat & 0xF8) | ((lyc == 0) << 2) | 2;
      stat_prev = (1 << 2) | ((lyc == 0) << 3);
      cycle_frame = 0;
      frames_done++;
    } else {
      while (cycle_frame >= CYCLES_PER_FRAME) {
        cycle_frame -= CYCLES_PER_FRAME;
        frames_done++;
        if (frames_done >= frames_to_run) break;
      }
    }
    delazify();
  }

  // One halted iteration (:976-1300), or a batch of them that no event can
  // interrupt. Exact state in and out.
  __device__ void halted_step(int frames_to_run) {
    const int lcdc_prev = lcdc & 0x80;
    int k = 1;
    if ((ie & iflag & 0x1F) == 0 && cycle_frame < CYCLES_PER_FRAME) {
      int kmax = (CYCLES_PER_FRAME - cycle_frame + 3) >> 2;  // iteration that ends the frame
      if (lcdc & 0x80) {
        // iteration that crosses a line the exact path must see (as in delazify)
        int to_line = CYCLES_PER_LINE - scan;
        if (!is_env0 && !(stat & 0x78))
          to_line += ((ly < SCREEN_H ? SCREEN_H : LINES_PER_FRAME) - 1 - ly) * CYCLES_PER_LINE;
        int kl = (to_line + 3) >> 2;
        kmax = kl < kmax ? kl : kmax;
      }
      if ((tac & 4) || rl_pending) {
        int t;
        if (rl_pending) {
          t = rl_delay;
        } else {
          int period = 1 << (div_bit(tac) + 1);
          t = period - (div & (period - 1)) + (0xFF - tima) * period + 4;
        }
        int kt = t <= 0 ? 1 : (t + 3) >> 2;                  // iteration of the next TIMA reload
        kmax = kt < kmax ? kt : kmax;
      }
      k = kmax - 1;
      if (k < 1) k = 1;
    }
    const int cycles = 4 * k;
    timer_tick(cycles);
    int lcdc_now = ppu_advance(cycles);
    const int pending = ie & iflag & 0x1F;
    int svc = 0;
    if (pending) {
      halted = 0;
      if (ime) {
        service(pending);
        svc = 20;
        timer_tick(20);
        lcdc_now = ppu_advance(20);
      } else {
        pc = (pc + 1) & 0xFFFF;  // :1181-1183
      }
    }
    const int total = cycles + svc;
    rtc_tick(total);
    cyc_run += total;
    cycle_frame += total;
    if (lcdc_prev && !(lcdc_now & 0x80)) {
      cycle_frame = 0;
      frames_done++;
      return;
    }
    while (cycle_frame >= CYCLES_PER_FRAME) {
      cycle_frame -= CYCLES_PER_FRAME;
      frames_done++;
      if (frames_done >= frames_to_run) break;
    }
  }

  // ---- out-of-line entry points of the interpreter loop ----------------------
  // They take `this` by address, so the cold state stays in local memory and
  // out of the loop's registers. Each is reached once per event, slow memory
  // access or fetch outside the window, not once per instruction.
  __device__ __noinline__ int read_slow(int a) { return read8(a); }
  __device__ __noinline__ void write_slow(int a, int v) { write8_slow(a & 0xFFFF, v); }
  // instruction bytes through the memory map (boot ROM overlay, RAM, bank
  // ends, banks outside the window)
  __device__ __noinline__ uint32_t fetch_slow(int at, const uint8_t* dec) {
    const int op = read8(at), b1 = read8((at + 1) & 0xFFFF), b2 = read8((at + 2) & 0xFFFF);
    const uint32_t e = op == 0xCB ? cb_family(b1) : dec[op];
    return (uint32_t)op | ((uint32_t)b1 << 8) | ((uint32_t)b2 << 16) | (e << 24);
  }
  // the exact tail of one instruction plus the halted iterations it leads
  // into; true when the launch's frames are done
  __device__ __noinline__ bool tail_slow(int cyc, int opcode, int pc_before, int frames_to_run) {
    slow_post(cyc, opcode, pc_before, frames_to_run);
    while (halted && frames_done < frames_to_run) {
      materialize();
      halted_step(frames_to_run);
      delazify();
    }
    return frames_done >= frames_to_run;
  }
  // unimplemented opcode (misc.py:42-56, kind 1) or a debug trap; the first
  // trap of an env keeps its pc, opcode and kind
  __device__ __noinline__ void trap_op(int at, int op, int kind) {
    if (trap) return;
    trap = 1;
    ev |= EV_TRAP;
    i32[(size_t)F_TRAP_PC * S] = at & 0xFFFF;
    i32[(size_t)F_TRAP_OPCODE * S] = op & 0xFF;
    i32[(size_t)F_TRAP_KIND * S] = kind;
  }
};

__device__ __forceinline__ int sign8(int v) { return v >= 128 ? v - 256 : v; }

// ---------------------------------------------------------------------------
// Uniform-datapath interpreter loop (gbx_udesc.h)
// ---------------------------------------------------------------------------
// Every lane runs the same stages for its own instruction: fetch, descriptor,
// operands, effective address, reads, adder / logic / rotate units, register,
// flag and memory results, PC, SP and cycles. Divergence is left to the
// memory operands (a branch taken by the lanes that have one), the accesses
// outside RAM (IO out of line; JOYP, banked ROM and cartridge registers
// inline in that branch), fetches outside the staged and switched-bank
// bytes, the special opcodes and the exact post-instruction tail. Same
// results, instruction for instruction, as the switch loop (both follow the
// reference templates).
// rom_s: raw bytes of ROM offsets [0, pre_s_words + 16) in shared memory as
// words; rom_g: the whole ROM (zero-padded by 16 bytes) as words; alive: the
// lanes of this warp that run an env (each must reach the loop's vote).
template <int MBC>
__device__ __forceinline__ void uniform_loop(Emu<MBC>& s, Hot& h, bool run, int& ninstr, int& win_hi,
                                             int& bankN_off, int& cram_off, const uint32_t* rom_s,
                                             const uint32_t* __restrict__ rom_g, int pre_s_words,
                                             const uint8_t* dec_s, const uint4* ud_s, const uint16_t* rot_s,
                                             int frames_to_run, unsigned alive) {
  uint8_t* const mem = s.mem;
  uint8_t* const cram = s.cart_ram;
  // Byte accesses: VRAM, WRAM, HRAM and the mapped cart-RAM bank inline, JOYP
  // from its register, everything else (IO, ROM, cartridge registers) out of
  // line through the full memory map.
  auto fast = [&](int a) {
    return ((a >> 13) | 2) == 6 || (unsigned)(a - 0xFF80) < 0x7Fu ||
           ((unsigned)(a - 0xA000) < 0x2000u && cram_off >= 0);
  };
  auto fptr = [&](int a) -> uint8_t* {
    return (unsigned)(a - 0xA000) < 0x2000u ? cram + (cram_off + a - 0xA000) : mem + a;
  };
  // JOYP in registers: its value and its value per select setting (the
  // out-of-line paths see them through s.joyp, synced around each call)
  int jp = s.joyp;
  uint32_t jtab = s.joyp_table();
  uint8_t* const jsel = s.u8s + (size_t)F_JOYP_SELECT * s.S;
  auto joyp_write = [&](int v) {
    jp = (int)((jtab >> ((v >> 1) & 0x18)) & 0xFF);
    *jsel = (uint8_t)(v & 0x30);
  };
  auto urd = [&](int a) -> int {  // full path
    if (fast(a)) return *fptr(a);
    if (a == 0xFF00) return jp;
    if (a < 0x8000) return s.rom_read(a);  // cartridge ROM, banked (no call)
    s.clk = h.clk;
    s.joyp = jp;
    return s.read_slow(a);
  };
  auto uwr = [&](int a, int v) {  // full path
    if (fast(a)) { *fptr(a) = (uint8_t)v; return; }
    if (a == 0xFF00) { joyp_write(v); return; }
    if (a < 0x8000) {  // cartridge registers: banking state only (no call, no timing)
      s.write_mbc(a, v);
      win_hi = s.win_hi; bankN_off = s.bankN_off; cram_off = s.cram_off;
      return;
    }
    s.clk = h.clk;
    s.joyp = jp;
    s.write_slow(a, v);
    jp = s.joyp;
    h.clk = s.clk;
    if (s.ev) h.next_ev = INT_MIN;
    win_hi = s.win_hi; bankN_off = s.bankN_off; cram_off = s.cram_off;
  };

  // Warp-synchronous loop: every live lane of the warp meets at the vote at
  // the end of each iteration, finished lanes included (their body is
  // skipped). Without this convergence point the lanes drift out of lockstep
  // when freshly restored envs are spread over the warps: on config 5 with 5 %
  // random restores per step the free loop issued 412 G warp instructions at
  // 14.7 active lanes against 318 G at 19.1 with the same restores packed into
  // the first warps (same emulated instructions); with the vote the step went
  // 566 -> 470 ms, at a 6 % cost (441 -> 470 ms) where no env is restored.
  for (;;) {
    if (run) {
    const int pc = h.pc;
    // ---- fetch: opcode and two operand bytes from the staged bytes or the
    //      switched bank (the two aligned words around them), else out of line
    uint32_t w;
    {
      const bool ins = (unsigned)pc < (unsigned)win_hi;
      const bool inn = (unsigned)(pc - 0x4000) < 0x3FFEu && bankN_off >= 0;
      const int idx = ins ? pc : pc + bankN_off;
      // both loads predicated, no branch between the staged and switched-bank
      // lanes (461 vs 470 ms on the config-5 bench step)
      const bool sm = ins || (inn && idx < pre_s_words);
      const bool gl = !sm && inn;
      const int wi = (sm || gl) ? (idx >> 2) : 0;
      uint32_t lo = 0, hi = 0;
      if (sm) { lo = rom_s[wi]; hi = rom_s[wi + 1]; }
      if (gl) { lo = __ldg(rom_g + wi); hi = __ldg(rom_g + wi + 1); }
      w = __funnelshift_r(lo, hi, (idx & 3) << 3);
      if (!(ins || inn)) { s.clk = h.clk; s.joyp = jp; w = s.fetch_slow(pc, dec_s); }
    }
    const int op = w & 0xFF, b1 = (w >> 8) & 0xFF, imm16 = (w >> 8) & 0xFFFF;
    const int key = op == 0xCB ? 256 + b1 : op;
    const uint4 q0 = ud_s[2 * key], q1 = ud_s[2 * key + 1];
    const uint32_t fa = q0.z, vx = q1.x, vy = q1.y;
    const int F = h.f;
    const bool taken = ((F ^ (int)(vy >> 8)) & (int)vy & 0xFF) == 0;
    // ---- operands and effective address ----
    const int A = h.A();
    const int xr = __byte_perm(h.bcde, h.hlxa, q0.x);
    const int pr = __byte_perm(h.bcde, h.hlxa, q0.x >> 16);
    const int p16 = (fa & UF_P_SP) ? h.sp : (pr | ((fa & UF_P_AF) ? F : 0));
    int ea = (fa & UF_EA_SP) ? h.sp : (int)__byte_perm(h.bcde, h.hlxa, q0.y);
    ea |= (fa & UF_EA_IMM16) ? imm16 : (fa & UF_EA_IMM8) ? b1 : 0;
    if (fa & UF_EA_FF) ea |= 0xFF00;
    ea = (ea - (int)((fa >> UF_EA_DEC_BIT) & 1)) & 0xFFFF;
    // ---- reads (the stack only when a conditional return is taken) ----
    const int ea1 = (ea + 1) & 0xFFFF;
    const bool rd1 = (fa & UF_RD1) && taken, rd2 = (fa & UF_RD2) && taken;
    int v0 = 0, v1 = 0;
    // memory operands through branches taken by the lanes that have one
    // (measured faster than issuing them predicated from the converged flow)
    if (rd1) {  // the second byte (POP, RET) only with the first
      v0 = urd(ea);
      if (rd2) v1 = urd(ea1);
    }
    const int x = (fa & UF_X_MEM) ? v0 : (fa & UF_X_IMM) ? b1 : xr;
    // ---- adder: 8-bit ALU, INC/DEC, 16-bit pair arithmetic ----
    const int k16 = (int)(q0.y >> 16);
    const int e8 = (b1 ^ 0x80) - 0x80;
    const int lsel = (vx >> UV_LSEL) & 3, rsel = (vx >> UV_RSEL) & 3;
    const int L = lsel == ULS_A ? A : lsel == ULS_X ? x : lsel == ULS_EA ? ea : p16;
    const int R = rsel == URS_X ? x : rsel == URS_K ? k16 : rsel == URS_P16 ? p16 : (e8 & 0xFFFF);
    const int sub = (fa >> UF_SUB_BIT) & 1;
    const int Rv = R ^ (sub ? 0xFF : 0);
    const int cin = (((fa & UF_CIN) ? (F >> 4) : 0) & 1) ^ sub;
    const int S = L + Rv + cin;
    const int cv = L ^ Rv ^ S;  // carries into each bit
    const bool wide = fa & UF_WIDE;
    const int ah = ((cv >> (wide ? 12 : 4)) & 1) ^ sub;
    const int ac = ((cv >> (wide ? 16 : 8)) & 1) ^ sub;
    // ---- logic: AND / OR / XOR (also BIT, RES, SET, CPL) ----
    const int P = (fa & UF_LX) ? x : A;
    const int Q = (fa & UF_QK) ? k16 : x;
    const int lop = (vx >> UV_LOP) & 3;
    const int la = P & Q, lo = P | Q;
    const int lres = lop == UL_AND ? la : lop == UL_OR ? lo : (lo ^ la);
    // ---- rotate / shift / swap: one lookup (kind, carry in, x) ----
    const uint32_t rv = rot_s[q1.z | ((F & 0x10) << 4) | x];
    const int rres = rv & 0xFF, rc = rv >> 8;
    // ---- 8-bit result and flags ----
    const int unit = (vx >> UV_UNIT) & 3;
    const int r8 = unit == UU_PASS ? x : unit == UU_ADD ? (S & 0xFF) : unit == UU_LOGIC ? lres : rres;
    const int hc = unit == UU_ADD ? ((ah << 5) | (ac << 4)) : unit == UU_ROT ? (rc << 4) : 0;
    const int fc = ((r8 == 0) << 7) | (sub << 6) | hc;
    const uint32_t fm = q0.w;  // keep | computed << 8 | set << 16 | xor << 24
    int Fn = (int)(((((uint32_t)F & fm) | ((uint32_t)fc & (fm >> 8)) | (fm >> 16)) ^ (fm >> 24)) & 0xF0);
    // ---- memory results (before the registers change: values and addresses
    //      come from the instruction's inputs) ----
    const int len = vx & 3;
    const int seq = pc + len;
    const int nw = (vx >> UV_NW) & 3;
    {
      const int vs = (vy >> UY_VSRC) & 3;
      const int val = vs == UVS_P16 ? p16 : vs == UVS_PCN ? (seq & 0xFFFF) : h.sp;
      const bool lof = fa & UF_LOFIRST;
      const int w0 = nw == 2 ? (lof ? (val & 0xFF) : (val >> 8)) : r8;
      const int w1 = lof ? (val >> 8) : (val & 0xFF);
      const int a1 = lof ? ea1 : ((ea - 1) & 0xFFFF);
      const bool wr0 = nw && taken, wr1 = nw == 2 && taken;
      if (wr0) {
        uwr(ea, w0);
        if (wr1) uwr(a1, w1);
      }
    }
    // ---- register results ----
    if (fa & UF_D8) {
      const int pos = (vx >> UV_D8POS) & 31;
      if (fa & UF_D8_HI) h.hlxa = Hot::insert_byte(h.hlxa, r8, pos);
      else h.bcde = Hot::insert_byte(h.bcde, r8, pos);
    }
    const int spd = (vy >> UY_SPD) & 3;  // 1: SP -= 2, 2: SP += 2
    if (spd && taken) h.sp = (h.sp + (spd == 1 ? -2 : 2)) & 0xFFFF;
    const int d16 = (vy >> UY_D16) & 7;
    if (d16) {
      const int r16 = (fa & UF_R16_POP) ? (v0 | (v1 << 8)) : (S & 0xFFFF);
      if (d16 == UD_SP) h.sp = r16;
      else if (d16 == UD_AF) { h.setA(r16 >> 8); Fn = r16 & 0xF0; }
      else if (d16 == UD_HL) h.hlxa = (h.hlxa & 0xFFFFu) | ((uint32_t)r16 << 16);
      else if (d16 == UD_BC) h.bcde = (h.bcde & 0xFFFFu) | ((uint32_t)r16 << 16);
      else h.bcde = (h.bcde & 0xFFFF0000u) | (uint32_t)r16;
    }
    h.f = Fn;
    // ---- next PC and cycles ----
    const int tsel = (vx >> UV_TSEL) & 7;
    int npc = seq;
    if (taken && tsel)
      npc = tsel == UT_IMM16 ? imm16 : tsel == UT_JR ? pc + 2 + e8 : tsel == UT_EA ? ea
          : tsel == UT_V16 ? (v0 | (v1 << 8)) : k16;
    int cyc = (int)((taken ? (vx >> UV_CYC_T) : (vx >> UV_CYC_NT)) & 15) << 2;
    // ---- special opcodes (misc.py, stack.py RETI, alu.py DAA) ----
    if (fa & UF_SPECIAL) {
      switch (op) {
        case 0x76: s.halted = 1; s.ev |= EV_HALT; h.next_ev = INT_MIN; break;
        case 0xF3: s.ime_delay = 0; s.ime = 0; break;
        case 0xFB: case 0xD9:  // EI, and RETI after its return
          s.ime_delay = 0;
          if (!s.ime) { s.ime = 1; s.ev |= EV_IRQ; h.next_ev = INT_MIN; }
          break;
        case 0x27: h.daa(); break;
        default:  // STOP and the unimplemented opcodes (misc.py:42-56)
          s.trap_op(pc, op, 1);
          h.next_ev = INT_MIN;
          npc = pc;
          cyc = 0;
          break;
      }
    }
    h.pc = npc & 0xFFFF;
    // ---- tail ----
    ninstr++;
    h.clk += cyc;
    bool stop = false;
    if (h.clk >= h.next_ev) {
      if (s.trap) {
        ninstr--;
        stop = true;
      } else {
        s.bcde = h.bcde; s.hlxa = h.hlxa; s.f = h.f; s.pc = h.pc; s.sp = h.sp; s.clk = h.clk;
        s.joyp = jp;
        stop = s.tail_slow(cyc, op, pc, frames_to_run);
        h.bcde = s.bcde; h.hlxa = s.hlxa; h.f = s.f; h.pc = s.pc; h.sp = s.sp; h.clk = s.clk;
        h.next_ev = s.next_ev;
        win_hi = s.win_hi; bankN_off = s.bankN_off; cram_off = s.cram_off;
        jp = s.joyp;
        jtab = s.joyp_table();  // the frame count may have crossed the release frame
      }
    }
    if (stop) run = false;
    }
    if (!__any_sync(alive, run)) break;
  }
  s.joyp = jp;
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
// K = envs per warp: lane l < K of global warp w runs env w*K + l (K = 1),
// or env 0 alone in warp 0 and env 1 + (w-1)*K + l in warp w >= 1. Small K
// spreads few envs over many warps (no divergence, more latency hiding);
// K = 32 packs a full warp (shared issue slots when envs run in lockstep).
// MAXT = largest block size the launch may use (caps registers at 64K/MAXT).
// DBG = the debug-trap instantiation (launched only when a trap is set).
// UNI = the uniform-datapath interpreter (gbx_udesc.h) in place of the
// per-family switch: for full warps of envs at different PCs.
// Shared memory, switch: pre-decoded words of ROM offsets [0, P) | boot ROM |
// family table. Uniform: raw ROM bytes [0, P + 16) | boot ROM | family table
// | descriptor table | rotate table. P = staged ROM offsets (pre_s_words).
__host__ __device__ constexpr size_t rom_smem_bytes(int P, bool uni) {
  return uni ? (((size_t)P + 16 + 15) & ~(size_t)15) : (size_t)P * 4;
}
__host__ __device__ constexpr size_t udesc_smem_offset(int P) { return rom_smem_bytes(P, true) + 512; }
// Env run by lane `lane` of global warp `gw` at K envs per warp, or -1.
// Env 0 alone takes the exact post-instruction path at every scanline (it
// records the scanline latches), so with K > 1 it gets warp 0 to itself and
// no other env waits on it; lane l < K of warp w >= 1 runs env 1 + (w-1)*K + l.
__device__ __forceinline__ int lane_env(int gw, int lane, int K, int n) {
  if (lane >= K) return -1;
  if (K > 1 && gw == 0 && lane != 0) return -1;
  const int env = K == 1 ? gw : gw == 0 ? 0 : 1 + (gw - 1) * K + lane;
  return env < n ? env : -1;
}

template <int MBC, int MAXT, bool DBG, bool UNI>
__global__ void __launch_bounds__(MAXT, 1)
    gb_step_kernel(DevState st, const uint32_t* __restrict__ pre_g, const int32_t* __restrict__ actions,
                   int frames_to_run, int release_after_frames, int stage, int K, int pre_s_words,
                   DebugCfg dbg) {
  extern __shared__ __align__(16) uint8_t smem[];
  uint32_t* pre_s = reinterpret_cast<uint32_t*>(smem);  // words (switch) or raw bytes (uniform)
  uint8_t* boot_s = smem + rom_smem_bytes(pre_s_words, UNI);
  uint8_t* dec_s = boot_s + 256;
  uint4* ud_s = reinterpret_cast<uint4*>(smem + udesc_smem_offset(pre_s_words));
  uint16_t* rot_s = reinterpret_cast<uint16_t*>(smem + udesc_smem_offset(pre_s_words) + sizeof(UDescTable));
  {
    const uint4* src = UNI ? reinterpret_cast<const uint4*>(st.rom) : reinterpret_cast<const uint4*>(pre_g);
    uint4* dst = reinterpret_cast<uint4*>(pre_s);
    const int n16 = (int)(rom_smem_bytes(pre_s_words, UNI) / 16);
    for (int k = threadIdx.x; k < n16; k += blockDim.x) dst[k] = __ldg(src + k);
    for (int k = threadIdx.x; k < 256; k += blockDim.x) {
      boot_s[k] = st.boot[k];
      dec_s[k] = c_decode.e[k];
    }
    if (UNI) {
      const uint4* ud = reinterpret_cast<const uint4*>(c_udesc.d);
      for (int k = threadIdx.x; k < UDESC_KEYS * 2; k += blockDim.x) ud_s[k] = ud[k];
      const uint4* rt = reinterpret_cast<const uint4*>(c_rot.v);
      uint4* rd = reinterpret_cast<uint4*>(rot_s);
      for (int k = threadIdx.x; k < (int)(sizeof(RotTable) / 16); k += blockDim.x) rd[k] = rt[k];
    }
  }
  __syncthreads();

  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int env = lane_env(gw, lane, K, st.n);
  if (env < 0) return;
  const size_t S = (size_t)st.S;

  Emu<MBC> s;
  s.mem = st.mem + (size_t)env * MEM_SIZE;
  s.S = st.S;
  s.pre_s = pre_s;
  s.pre_g = pre_g;
  s.boot_s = boot_s;
  s.rom_g = st.rom;
  s.cart_state = st.cart_state + env;
  s.cart_ram = st.cart_ram + (size_t)env * st.ram_rows;
  s.serial = st.serial + (size_t)env * SERIAL_MAX;
  s.i32 = st.i32 + env;
  s.u8s = st.u8s + env;
  s.latch = st.latch;
  s.rom_bank_count = st.rom_bank_count;
  s.rom_bank_mask = st.rom_bank_mask;
  s.ram_bank_count = st.ram_bank_count;
  s.pre_s_words = pre_s_words;
  s.is_env0 = env == 0;

  const int32_t* I = st.i32 + env;
  auto ld = [&](int fld) { return I[(size_t)fld * S]; };
  s.pc = ld(F_PC) & 0xFFFF;
  s.sp = ld(F_SP) & 0xFFFF;
  s.bcde = ((uint32_t)(ld(F_B) & 0xFF) << 24) | ((uint32_t)(ld(F_C) & 0xFF) << 16) |
           ((uint32_t)(ld(F_D) & 0xFF) << 8) | (uint32_t)(ld(F_E) & 0xFF);
  s.hlxa = ((uint32_t)(ld(F_H) & 0xFF) << 24) | ((uint32_t)(ld(F_L) & 0xFF) << 16) | (uint32_t)(ld(F_A) & 0xFF);
  s.f = ld(F_F) & 0xF0;
  s.cycle_frame = ld(F_CYCLE_IN_FRAME);
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
  s.cyc_run = 0;
  s.ninstr = 0;
  // state is exact (lazy == 0) until the first exact tail has run
  s.lazy = 0;
  s.ev = EV_FIRST;
  s.clk = 0;
  s.next_ev = INT_MAX;
  s.stat_hi = s.stat & 0xF8;
  s.lcd_on = 0;
  s.rtc_run = 0;
  s.lcdc_before = s.lcdc;

  bool run = s.frames_done < frames_to_run && !s.trap;
  // a halted start runs the halted loop first
  if (run && s.halted) {
    while (s.halted && s.frames_done < frames_to_run) s.halted_step(frames_to_run);
    run = s.frames_done < frames_to_run;
  }

  // watched byte at launch start (cpu_step_builder.py:948-951)
  const int watch_val = (DBG && dbg.watch_addr) ? s.raw_read(dbg.watch_addr & 0xFFFF) : 0;

  // ---- interpreter loop: registers in h, cold state in s ----
  Hot h;
  h.bcde = s.bcde; h.hlxa = s.hlxa; h.f = s.f; h.pc = s.pc; h.sp = s.sp;
  h.clk = 0;
  h.next_ev = INT_MIN;  // EV_FIRST: the first instruction takes the exact tail
  int ninstr = 0;
  int win_hi = s.win_hi, bankN_off = s.bankN_off, cram_off = s.cram_off;
  uint8_t* const mem = s.mem;
  uint8_t* const cram = s.cart_ram;
  auto save = [&]() {
    s.bcde = h.bcde; s.hlxa = h.hlxa; s.f = h.f; s.pc = h.pc; s.sp = h.sp; s.clk = h.clk;
  };
  auto load = [&]() {
    h.bcde = s.bcde; h.hlxa = s.hlxa; h.f = s.f; h.pc = s.pc; h.sp = s.sp; h.clk = s.clk;
    h.next_ev = s.next_ev;
    win_hi = s.win_hi; bankN_off = s.bankN_off; cram_off = s.cram_off;
  };
  // VRAM, WRAM and HRAM are plain bytes of the env's address space
  auto plain = [](int a) { return ((a >> 13) | 2) == 6 || (unsigned)(a - 0xFF80) < 0x7Fu; };
  auto rd = [&](int a) -> int {
    if (plain(a)) return mem[a];
    if ((unsigned)(a - 0xA000) < 0x2000u && cram_off >= 0) return cram[cram_off + a - 0xA000];
    if (a == 0xFF00) return s.joyp;  // JOYP: no clock, no side effect
    s.clk = h.clk;  // lazy DIV/TIMA/STAT/LY reads need the clock
    return s.read_slow(a);
  };
  auto wr = [&](int a, int v) {
    if (plain(a)) { mem[a] = (uint8_t)v; return; }
    if ((unsigned)(a - 0xA000) < 0x2000u && cram_off >= 0) { cram[cram_off + a - 0xA000] = (uint8_t)v; return; }
    if (a == 0xFF00) { s.write_joyp(v); return; }  // JOYP select: no event, no sync
    s.clk = h.clk;
    s.write_slow(a, v);  // ev is 0 here unless an earlier write of this instruction set it
    h.clk = s.clk;       // a timing write syncs (clk = 0) and sets ev
    if (s.ev) h.next_ev = INT_MIN;
    win_hi = s.win_hi; bankN_off = s.bankN_off; cram_off = s.cram_off;
  };

  if constexpr (UNI) {
    // lanes of this warp that run an env (the others returned above)
    unsigned alive = 0;
    for (int l = 0; l < K; l++)
      if (lane_env(gw, l, K, st.n) >= 0) alive |= 1u << l;
    uniform_loop<MBC>(s, h, run, ninstr, win_hi, bankN_off, cram_off, pre_s,
                      reinterpret_cast<const uint32_t*>(st.rom), pre_s_words, dec_s, ud_s, rot_s, frames_to_run,
                      alive);
  } else while (run) {
    // ---- fetch + decode ----
    const int pc = h.pc;
    uint32_t w;
    if ((unsigned)pc < (unsigned)win_hi) {
      w = pre_s[pc];
    } else if ((unsigned)(pc - 0x4000) < 0x3FFEu && bankN_off >= 0) {
      const int idx = pc + bankN_off;
      w = idx < pre_s_words ? pre_s[idx] : __ldg(pre_g + idx);
    } else {
      s.clk = h.clk;
      w = s.fetch_slow(pc, dec_s);
    }
    const int opcode = w & 0xFF;
    const int fam = w >> 24;
    // Operand fields are extracted inside the cases that use them: hoisted
    // above the switch they cost every instruction (NOP 55 -> 49 warp
    // instructions without them).
#define IMM8 ((int)((w >> 8) & 0xFF))
#define IMM16 ((int)((w >> 8) & 0xFFFF))
#define YF ((opcode >> 3) & 7)
#define ZF (opcode & 7)
    if (DBG) {  // checks before execution (:1320-1338)
      if (dbg.trap_pc && pc == dbg.trap_pc) { s.trap_op(pc, opcode, 5); break; }
      if (dbg.trap_rst38 && opcode == 0xFF && pc != 0x0038) { s.trap_op(pc, opcode, 3); break; }
    }
    // Memory operands are read inside the families that have them (reads
    // have no side effects, so RET cc reads the stack only when taken).
    // ---- execute ----
    int npc = pc + 1;
    int cyc = 4;
    int nw = 0, wa0, wv0, wa1, wv1;  // the slots are read only below nw
    switch (fam) {
      case FM_LDRR: h.setr(YF, h.getr(ZF)); break;  // includes NOP (LD B,B form)
      case FM_LD16: h.setp((opcode >> 4) & 3, IMM16); npc = pc + 3; cyc = 12; break;
      case FM_ST_A:
        nw = 1; wv0 = h.A();
        if (opcode < 0x40) {
          const int p = (opcode >> 4) & 3;  // 0 BC, 1 DE, 2 HL+, 3 HL-
          const int ad = p == 0 ? h.BC() : p == 1 ? h.DE() : h.HL();
          wa0 = ad;
          if (p >= 2) h.setHL(p == 2 ? ad + 1 : ad - 1);
          cyc = 8;
        } else if (opcode == 0xE0) { wa0 = 0xFF00 | IMM8; npc = pc + 2; cyc = 12; }
        else if (opcode == 0xE2) { wa0 = 0xFF00 | h.C_(); cyc = 8; }
        else { wa0 = IMM16; npc = pc + 3; cyc = 16; }
        break;
      case FM_LD_A:
        if (opcode < 0x40) {
          const int p = (opcode >> 4) & 3;  // 0 BC, 1 DE, 2 HL+, 3 HL-
          const int ad = p == 0 ? h.BC() : p == 1 ? h.DE() : h.HL();
          h.setA(rd(ad));
          if (p >= 2) h.setHL(p == 2 ? ad + 1 : ad - 1);
          cyc = 8;
        } else if (opcode == 0xF0) { h.setA(rd(0xFF00 | IMM8)); npc = pc + 2; cyc = 12; }
        else if (opcode == 0xF2) { h.setA(rd(0xFF00 | h.C_())); cyc = 8; }
        else { h.setA(rd(IMM16)); npc = pc + 3; cyc = 16; }
        break;
      case FM_INCDEC16: {
        const int p = (opcode >> 4) & 3;
        h.setp(p, h.getp(p) + ((opcode & 8) ? -1 : 1));
        cyc = 8; break;
      }
      case FM_INCDEC8: {
        const int dec1 = ZF & 1;
        const int old = h.getr(YF), v = (dec1 ? old - 1 : old + 1) & 0xFF;
        h.setr(YF, v);
        h.f = FLAGS(v == 0, dec1, dec1 ? (old & 0xF) == 0 : (old & 0xF) == 0xF, (h.f >> 4) & 1);
        break;
      }
      case FM_INCDEC_HL: {
        const int old = rd(h.HL()), dec1 = ZF & 1;
        const int v = (dec1 ? old - 1 : old + 1) & 0xFF;
        h.f = FLAGS(v == 0, dec1, dec1 ? (old & 0xF) == 0 : (old & 0xF) == 0xF, (h.f >> 4) & 1);
        nw = 1; wa0 = h.HL(); wv0 = v;
        cyc = 12; break;
      }
      case FM_LD8_IMM: h.setr(YF, IMM8); npc = pc + 2; cyc = 8; break;
      case FM_ST_HL_IMM: nw = 1; wa0 = h.HL(); wv0 = IMM8; npc = pc + 2; cyc = 12; break;
      case FM_ROTA: {
        const int a = h.A(), oc = (h.f >> 4) & 1;
        const int right = YF & 1, thru = YF >> 1;
        const int c = right ? (a & 1) : ((a >> 7) & 1);
        const int in = thru ? oc : c;
        const int r = right ? ((a >> 1) | (in << 7)) : (((a << 1) & 0xFF) | in);
        h.setA(r); h.f = FLAGS(0, 0, 0, c);
        break;
      }
      case FM_ST_SP16:
        nw = 2; wa0 = IMM16; wv0 = h.sp & 0xFF; wa1 = (IMM16 + 1) & 0xFFFF; wv1 = (h.sp >> 8) & 0xFF;
        npc = pc + 3; cyc = 20; break;
      case FM_ADDHL: {
        const int hl = h.HL(), rr = h.getp((opcode >> 4) & 3), sum = hl + rr;
        h.f = FLAGS((h.f >> 7) & 1, 0, ((hl & 0xFFF) + (rr & 0xFFF)) > 0xFFF, sum > 0xFFFF);
        h.setHL(sum);
        cyc = 8; break;
      }
      case FM_JR: {
        const bool t = opcode == 0x18 || h.cond(YF);
        npc = pc + 2 + (t ? sign8(IMM8) : 0);
        cyc = t ? 12 : 8;
        break;
      }
      case FM_DAA: h.daa(); break;
      case FM_FLAGOP: {  // CPL (YF=5), SCF (YF=6), CCF (YF=7)
        const int zf = (h.f >> 7) & 1, cf = (h.f >> 4) & 1;
        if (YF == 5) { h.setA(h.A() ^ 0xFF); h.f = FLAGS(zf, 1, 1, cf); }
        else h.f = FLAGS(zf, 0, 0, YF == 6 ? 1 : !cf);
        break;
      }
      case FM_LDR_HL: h.setr(YF, rd(h.HL())); cyc = 8; break;
      case FM_STHL_R: nw = 1; wa0 = h.HL(); wv0 = h.getr(ZF); cyc = 8; break;
      case FM_HALT: s.halted = 1; s.ev |= EV_HALT; h.next_ev = INT_MIN; break;
      case FM_ALU_ADC: {  // ADD, ADC (alu.py)
        const int a = h.A(), v = h.getr(ZF), cin = YF & (h.f >> 4) & 1, r = a + v + cin;
        h.f = (((r & 0xFF) == 0) << 7) | ((((a & 0xF) + (v & 0xF) + cin) > 0xF) << 5) | ((r > 0xFF) << 4);
        h.setA(r);
        break;
      }
      case FM_ALU_SBC: {  // SUB, SBC, CP
        const int a = h.A(), v = h.getr(ZF), cin = YF == 3 ? (h.f >> 4) & 1 : 0, r = a - v - cin;
        h.f = (((r & 0xFF) == 0) << 7) | 0x40 | ((((a & 0xF) - (v & 0xF) - cin) < 0) << 5) | ((r < 0) << 4);
        if (YF != 7) h.setA(r);
        break;
      }
      case FM_ALU_LOG: {  // AND, XOR, OR
        const int a = h.A(), v = h.getr(ZF);
        const int r = YF == 4 ? (a & v) : YF == 5 ? (a ^ v) : (a | v);
        h.f = ((r == 0) << 7) | (YF == 4 ? 0x20 : 0);
        h.setA(r);
        break;
      }
      case FM_ALU_V: {
        const bool hl = opcode < 0xC0;  // ALU A,(HL); else ALU A,d8
        h.alu(YF, hl ? rd(h.HL()) : IMM8);
        npc = pc + (hl ? 1 : 2);
        cyc = 8; break;
      }
      case FM_RET:
        if (opcode == 0xC9 || opcode == 0xD9 || h.cond(YF)) {
          npc = rd(h.sp) | (rd((h.sp + 1) & 0xFFFF) << 8);
          h.sp = (h.sp + 2) & 0xFFFF;
          if (opcode == 0xD9) {
            s.ime_delay = 0;
            // Setting IME can make a pending interrupt serviceable; with IME
            // already set none is pending (every IF/IE change is an event).
            if (!s.ime) { s.ime = 1; s.ev |= EV_IRQ; h.next_ev = INT_MIN; }
          }
          cyc = (opcode & 1) ? 16 : 20;
        } else {
          cyc = 8;
        }
        break;
      case FM_POP: {
        const int p = (opcode >> 4) & 3;
        const int v1 = rd(h.sp), v2 = rd((h.sp + 1) & 0xFFFF);
        if (p == 3) { h.setA(v2); h.f = v1 & 0xF0; }
        else h.setp(p, v1 | (v2 << 8));
        h.sp = (h.sp + 2) & 0xFFFF;
        cyc = 12; break;
      }
      case FM_JP:
        if (opcode == 0xE9) { npc = h.HL(); break; }
        {
          const bool t = opcode == 0xC3 || h.cond(YF);
          npc = t ? IMM16 : pc + 3;
          cyc = t ? 16 : 12;
        }
        break;
      case FM_CALL:
        if (opcode == 0xCD || h.cond(YF)) {
          const int ret = (pc + 3) & 0xFFFF;
          nw = 2; wa0 = (h.sp - 1) & 0xFFFF; wv0 = ret >> 8; wa1 = (h.sp - 2) & 0xFFFF; wv1 = ret & 0xFF;
          h.sp = (h.sp - 2) & 0xFFFF;
          npc = IMM16; cyc = 24;
        } else {
          npc = pc + 3; cyc = 12;
        }
        break;
      case FM_PUSH: {
        const int p = (opcode >> 4) & 3;
        const int v = p == 3 ? ((h.A() << 8) | (h.f & 0xF0)) : h.getp(p);
        nw = 2; wa0 = (h.sp - 1) & 0xFFFF; wv0 = v >> 8; wa1 = (h.sp - 2) & 0xFFFF; wv1 = v & 0xFF;
        h.sp = (h.sp - 2) & 0xFFFF;
        cyc = 16; break;
      }
      case FM_RST: {
        const int ret = (pc + 1) & 0xFFFF;
        nw = 2; wa0 = (h.sp - 1) & 0xFFFF; wv0 = ret >> 8; wa1 = (h.sp - 2) & 0xFFFF; wv1 = ret & 0xFF;
        h.sp = (h.sp - 2) & 0xFFFF;
        npc = opcode & 0x38; cyc = 16; break;
      }
      // CB-prefixed (bitops.py): RLC RRC RL RR SLA SRA SWAP SRL, BIT, RES, SET
      case FM_CB_ROT: {
        const int cz = IMM8 & 7;
        int c;
        const int res = cb_rot((IMM8 >> 3) & 7, h.getr(cz), (h.f >> 4) & 1, c);
        h.f = ((res == 0) << 7) | (c << 4);
        h.setr(cz, res);
        npc = pc + 2; cyc = 8; break;
      }
      case FM_CB_BIT:  // Z from the bit, H set, C kept
        h.f = ((((h.getr(IMM8 & 7) >> ((IMM8 >> 3) & 7)) & 1) ^ 1) << 7) | 0x20 | (h.f & 0x10);
        npc = pc + 2; cyc = 8; break;
      case FM_CB_RES: {
        const int cz = IMM8 & 7;
        h.setr(cz, h.getr(cz) & ~(1 << ((IMM8 >> 3) & 7)));
        npc = pc + 2; cyc = 8; break;
      }
      case FM_CB_SET: {
        const int cz = IMM8 & 7;
        h.setr(cz, h.getr(cz) | (1 << ((IMM8 >> 3) & 7)));
        npc = pc + 2; cyc = 8; break;
      }
      case FM_CB_HL: {  // the (HL) forms
        const int cy = (IMM8 >> 3) & 7, grp = IMM8 >> 6, v = rd(h.HL());
        npc = pc + 2;
        if (grp == 1) {
          h.f = ((((v >> cy) & 1) ^ 1) << 7) | 0x20 | (h.f & 0x10);
          cyc = 12;
          break;
        }
        int res;
        if (grp == 0) {
          int c;
          res = cb_rot(cy, v, (h.f >> 4) & 1, c);
          h.f = ((res == 0) << 7) | (c << 4);
        } else {
          res = grp == 2 ? (v & ~(1 << cy) & 0xFF) : (v | (1 << cy));
        }
        nw = 1; wa0 = h.HL(); wv0 = res; cyc = 16;
        break;
      }
      case FM_SPADD:
        if (opcode == 0xF9) { h.sp = h.HL(); cyc = 8; break; }
        {
          const int ou = IMM8, res = (h.sp + sign8(IMM8)) & 0xFFFF;
          h.f = FLAGS(0, 0, ((h.sp & 0xF) + (ou & 0xF)) > 0xF, ((h.sp & 0xFF) + ou) > 0xFF);
          if (opcode == 0xE8) { h.sp = res; cyc = 16; }
          else { h.setHL(res); cyc = 12; }
          npc = pc + 2;
        }
        break;
      case FM_IME:  // EI, DI (misc.py); EI with IME already set changes nothing (see RETI)
        s.ime_delay = 0;
        if (opcode == 0xFB) {
          if (!s.ime) { s.ime = 1; s.ev |= EV_IRQ; h.next_ev = INT_MIN; }
        } else {
          s.ime = 0;
        }
        break;
      default:  // FM_TRAP (misc.py:42-56)
        s.trap_op(pc, opcode, 1);
        h.next_ev = INT_MIN;
        npc = pc;
        cyc = 0;
        break;
    }
#undef IMM8
#undef IMM16
#undef YF
#undef ZF
    h.pc = npc & 0xFFFF;
    // ---- memory writes ----
    if (nw) {
      wr(wa0, wv0);
      if (nw == 2) wr(wa1, wv1);
    }
    // ---- tail ----
    ninstr++;
    if (DBG) {  // checks after execution (:1362-1393); a trapping instruction's cycles never run
      if (dbg.trap_rst38 && h.pc >= 0xFE00) { s.trap_op(pc, opcode, 4); ninstr--; break; }
      if (s.trap) { ninstr--; break; }
      if (dbg.max_instr > 0 && ninstr >= dbg.max_instr) { s.trap_op(h.pc, opcode, 6); break; }
      if (dbg.watch_addr) {
        const int a = dbg.watch_addr & 0xFFFF;
        s.clk = h.clk;
        if (s.raw_read(a) != watch_val) { s.trap_op(pc, opcode, 7); break; }
      }
    }
    h.clk += cyc;
    if (h.clk >= h.next_ev) {
      if (s.trap) { ninstr--; break; }
      save();
      const bool done = s.tail_slow(cyc, opcode, pc, frames_to_run);
      load();
      if (done) break;
    }
  }
  if (run) save();
  s.ninstr = ninstr;
  s.sync_all();

  // ---- post-step body (post_step.py:11-102) ----
  const int a = s.hlxa & 0xFF, b = (s.bcde >> 24) & 0xFF, c = (s.bcde >> 16) & 0xFF, d = (s.bcde >> 8) & 0xFF;
  const int e_ = s.bcde & 0xFF, hh = (s.hlxa >> 24) & 0xFF, l = (s.hlxa >> 16) & 0xFF;
  if (stage == STAGE_OBS || stage == STAGE_FULL) {
    float* o = st.obs + (size_t)env * OBS_DIM;
    int m[16];
    {
      const uint4 q16 = *reinterpret_cast<const uint4*>(&s.M(0xC000));  // 16-byte aligned
      const uint32_t w4[4] = {q16.x, q16.y, q16.z, q16.w};
#pragma unroll
      for (int k = 0; k < 16; k++) m[k] = (w4[k >> 2] >> (8 * (k & 3))) & 0xFF;
    }
    float4 q[8];
    q[0] = make_float4((float)(s.pc & 0xFFFF) / 65535.0f, (float)(s.sp & 0xFFFF) / 65535.0f,
                       (float)a / 255.0f, (float)(s.f & 0xFF) / 255.0f);
    q[1] = make_float4((float)b / 255.0f, (float)c / 255.0f, (float)d / 255.0f, (float)e_ / 255.0f);
    q[2] = make_float4((float)hh / 255.0f, (float)l / 255.0f, (float)m[0] / 255.0f, (float)m[1] / 255.0f);
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
  stv(F_A, a); stv(F_B, b); stv(F_C, c); stv(F_D, d); stv(F_E, e_); stv(F_H, hh); stv(F_L, l);
  stv(F_F, s.f & 0xF0);
  stv(F_CYCLE_IN_FRAME, s.cycle_frame);
  stv(F_TRAP_FLAG, s.trap);
  stv(F_IME, s.ime); stv(F_IME_DELAY, s.ime_delay); stv(F_HALTED, s.halted);
  stv(F_DIV_COUNTER, s.div); stv(F_TIMER_PREV_IN, s.prev_in);
  stv(F_TIMA_RELOAD_PENDING, s.rl_pending); stv(F_TIMA_RELOAD_DELAY, s.rl_delay);
  stv(F_PPU_SCANLINE_CYCLE, s.scan); stv(F_PPU_LY, s.ly); stv(F_PPU_WINDOW_LINE, s.wl);
  st.u8s[(size_t)F_STAT_PREV * S + env] = (uint8_t)s.stat_prev;
  st.i64[(size_t)F_INSTR_COUNT * S + env] += s.ninstr;
  st.i64[(size_t)F_CYCLE_COUNT * S + env] += s.cyc_run;
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
static int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return v && *v ? atoi(v) : dflt;
}

// Largest number of this kernel's warps one SM holds: one block per SM (the
// staged ROM fills most of shared memory) of at most 1024 threads.
constexpr int WARPS_PER_SM = 32;

// Envs per warp that fills the GPU with one wave of warps: the smallest K in
// {1, 2, 4, 8, 16, 32} with ceil(n / K) <= sms * WARPS_PER_SM. A warp's time
// per step is set by the dependent chain of its interpreter loop and grows
// only slowly with the warps sharing its SM, so one full wave of warps
// beats both fewer, fuller warps and a second wave. Measured on B200
// (config-4 cartridge, frameskip 24): 65,536 envs 479 ms at K = 16 vs 522 ms
// at K = 32 and 713 ms at K = 8; 16,384 envs 233 ms at K = 4 vs 326 ms at
// K = 1 and 456 ms at K = 32. A HALT-heavy program can prefer K = 32 instead
// (config 3 at 16,384 envs: 25-44 ms at K = 32, 64-112 ms at K = 4), which is
// why the caller times the candidates on its first steps.
int fill_envs_per_warp(long long n, int sms) {
  const long long slots = (long long)(sms > 0 ? sms : 1) * WARPS_PER_SM;
  int k = 1;
  while (k < 32 && (n + k - 1) / k > slots) k <<= 1;
  return k;
}

// GBX_ENVS_PER_WARP (1..32) fixes K for every handle; 0 or unset = automatic.
int envs_per_warp_override() {
  const int k = env_int("GBX_ENVS_PER_WARP", 0);
  return k <= 0 ? 0 : k > 32 ? 32 : k;
}

// GBX_DISPATCH=switch or =uniform fixes the interpreter for every handle
// (gbx_dispatch values 1 and 2); unset or anything else = automatic.
int dispatch_override() {
  const char* v = getenv("GBX_DISPATCH");
  if (!v) return 0;
  if (!strcmp(v, "switch")) return 1;
  if (!strcmp(v, "uniform")) return 2;
  return 0;
}

template <int MBC, int MAXT, bool DBG, bool UNI = false>
static cudaError_t launch_t(const DevState& st, const uint32_t* pre, const int32_t* actions, int frames,
                            int release, int stage, cudaStream_t stream, int K, int threads, int blocks,
                            int pre_s_words, size_t sm, const DebugCfg& dbg) {
  cudaError_t e = cudaFuncSetAttribute(gb_step_kernel<MBC, MAXT, DBG, UNI>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  if (e != cudaSuccess) return e;
  gb_step_kernel<MBC, MAXT, DBG, UNI><<<blocks, threads, sm, stream>>>(st, pre, actions, frames, release, stage,
                                                                      K, pre_s_words, dbg);
  return cudaGetLastError();
}

template <int MBC>
static cudaError_t launch_mbc(const DevState& st, const uint32_t* pre, const int32_t* actions, int frames,
                              int release, int stage, cudaStream_t stream, const DebugCfg& dbg, int K,
                              int sms, bool uniform) {
  K = K < 1 ? 1 : K > 32 ? 32 : K;
  sms = sms < 1 ? 1 : sms;
  const long long warps = K == 1 ? st.n : 1 + (st.n - 1 + K - 1) / K;  // env 0 in a warp of its own
  // one block per SM (the pre-decoded banks fill shared memory): spread warps
  int per_block = (int)((warps + sms - 1) / sms);
  per_block = per_block < 1 ? 1 : per_block > WARPS_PER_SM ? WARPS_PER_SM : per_block;
  const int threads = per_block * 32;
  const int blocks = (int)((warps + per_block - 1) / per_block);
  int stage_words = env_int("GBX_ROM_SMEM_WORDS", ROM_SMEM_MAX);  // experiments: staged ROM size
  stage_words = stage_words < 0x400 ? 0x400 : stage_words > 0x8000 ? 0x8000 : stage_words & ~0xFF;
  const int rom_words = st.rom_bytes < stage_words ? st.rom_bytes : stage_words;
  const size_t sm = (size_t)rom_words * 4 + 512;
  if (dbg.active())  // debug traps: one instantiation (its 64-register bound fits every block size)
    return launch_t<MBC, 1024, true>(st, pre, actions, frames, release, stage, stream, K, threads, blocks,
                                     rom_words, sm, dbg);
  if (uniform)  // one instantiation: the 64-register bound fits every block size
    return launch_t<MBC, 1024, false, true>(st, pre, actions, frames, release, stage, stream, K, threads,
                                            blocks, rom_words,
                                            udesc_smem_offset(rom_words) + sizeof(UDescTable) + sizeof(RotTable),
                                            dbg);
  if (threads <= 256)
    return launch_t<MBC, 256, false>(st, pre, actions, frames, release, stage, stream, K, threads, blocks,
                                     rom_words, sm, dbg);
  if (threads <= 512)
    return launch_t<MBC, 512, false>(st, pre, actions, frames, release, stage, stream, K, threads, blocks,
                                     rom_words, sm, dbg);
  return launch_t<MBC, 1024, false>(st, pre, actions, frames, release, stage, stream, K, threads, blocks,
                                    rom_words, sm, dbg);
}

// K = envs per warp (1..32), sms = the device's SM count, uniform = the
// uniform-datapath interpreter instead of the switch (ignored while debug
// traps are set).
cudaError_t launch_step(const DevState& st, const uint32_t* pre, const int32_t* actions, int frames, int release,
                        int stage, cudaStream_t stream, const DebugCfg& dbg, int K, int sms, bool uniform) {
  switch (st.mbc_kind) {
    case MBC_MBC1:
      return launch_mbc<MBC_MBC1>(st, pre, actions, frames, release, stage, stream, dbg, K, sms, uniform);
    case MBC_MBC3:
      return launch_mbc<MBC_MBC3>(st, pre, actions, frames, release, stage, stream, dbg, K, sms, uniform);
    default:
      return launch_mbc<MBC_ROM_ONLY>(st, pre, actions, frames, release, stage, stream, dbg, K, sms, uniform);
  }
}

}  // namespace gbx
