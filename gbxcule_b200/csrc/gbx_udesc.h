// gbx_udesc.h - per-opcode descriptors of the uniform-datapath interpreter.
//
// The uniform interpreter (gb_step_kernel<..., UNI = true>) runs every SM83
// instruction through ONE fixed sequence of datapath stages, so that the 32
// lanes of a warp, each emulating its own console at its own PC, issue the
// same instructions every iteration and never split into per-opcode branches.
// Each stage is steered per lane by a 32-byte descriptor of the instruction,
// looked up by key = opcode (0..255) or 256 + second byte for the CB-prefixed
// opcodes:
//
//   operands  x     = a register (byte-permute selector), the immediate byte
//                     or the byte read at the effective address
//             p16   = a register pair (selector), SP, or AF
//   address   ea    = pair | SP | immediate (8/16-bit) | 0xFF00, minus 1 for
//                     the pushes; up to two bytes read at ea, ea + 1
//   units     adder L + R (+carry) with 8- or 16-bit half/full carry taps;
//             logic (AND / OR / XOR of A-or-x with x-or-constant);
//             rotate/shift/swap of x (one lookup in a 4096-entry table)
//   results   8-bit register, 16-bit pair (BC DE HL SP AF), memory (one byte
//             at ea or a 16-bit value as two bytes), flags by keep / computed
//             / set / xor masks, SP += 0 / -2 / +2, PC from the sequential
//             address or a target (imm16, JR, ea, popped word, RST vector),
//             cycles taken / not taken by the condition
//
// Semantics are those of the switch interpreter in gbx_step.cu (itself
// following src/gbxcule/kernels/cpu_templates/*.py); the descriptor only
// re-expresses each opcode's template as a setting of the common stages.
// DAA, HALT, DI, EI, the IME half of RETI and the trapping opcodes are
// marked special and finished by a small out-of-datapath switch.
#pragma once
#include <stdint.h>

namespace gbx {

// byte-permute selectors over {bcde, hlxa} (bytes E D C B | A 0 L H)
constexpr uint32_t PS_ZERO = 0x5555, PS_BC = 0x5532, PS_DE = 0x5510, PS_HL = 0x5576, PS_AHI = 0x5545,
                   PS_C = 0x5552;
__host__ __device__ constexpr uint32_t ps_reg(int r) { return (uint32_t)((r ^ 3) | 0x5550); }

// q0.z flag bits
enum UFlag : uint32_t {
  UF_EA_SP = 1u << 0, UF_EA_IMM8 = 1u << 1, UF_EA_IMM16 = 1u << 2, UF_EA_FF = 1u << 3, UF_EA_DEC = 1u << 4,
  UF_RD1 = 1u << 5, UF_RD2 = 1u << 6, UF_X_MEM = 1u << 7, UF_X_IMM = 1u << 8, UF_P_SP = 1u << 9,
  UF_P_AF = 1u << 10, UF_SUB = 1u << 11, UF_CIN = 1u << 12, UF_WIDE = 1u << 13, UF_SPECIAL = 1u << 14,
  UF_R16_POP = 1u << 15, UF_LOFIRST = 1u << 16, UF_D8 = 1u << 19,
  UF_D8_HI = 1u << 20, UF_LX = 1u << 21, UF_QK = 1u << 22
};
constexpr int UF_SUB_BIT = 11, UF_EA_DEC_BIT = 4;

// q1.x value fields
constexpr int UV_LEN = 0;      // 2 bits
constexpr int UV_CYC_NT = 2;   // 4 bits, cycles / 4
constexpr int UV_CYC_T = 6;    // 4 bits, cycles / 4
constexpr int UV_D8POS = 10;   // 5 bits: bit position of the 8-bit destination in its word
constexpr int UV_UNIT = 16;    // 2 bits
constexpr int UV_LOP = 18;     // 2 bits
constexpr int UV_LSEL = 20;    // 2 bits
constexpr int UV_RSEL = 22;    // 2 bits
constexpr int UV_TSEL = 26;    // 3 bits
constexpr int UV_NW = 29;      // 2 bits
// q1.y: [7:0] condition flag mask, [15:8] value that flag must have, then
constexpr int UY_D16 = 16;     // 3 bits
constexpr int UY_VSRC = 19;    // 2 bits
constexpr int UY_SPD = 21;     // 2 bits

enum UUnit { UU_PASS = 0, UU_ADD = 1, UU_LOGIC = 2, UU_ROT = 3 };
enum ULop { UL_AND = 0, UL_OR = 1, UL_XOR = 2 };
enum ULsel { ULS_A = 0, ULS_X = 1, ULS_EA = 2, ULS_P16 = 3 };
enum URsel { URS_X = 0, URS_K = 1, URS_P16 = 2, URS_E8 = 3 };
enum UTsel { UT_SEQ = 0, UT_IMM16 = 1, UT_JR = 2, UT_EA = 3, UT_V16 = 4, UT_K = 5 };
enum UD16 { UD_NONE = 0, UD_BC = 1, UD_DE = 2, UD_HL = 3, UD_SP = 4, UD_AF = 5 };
enum UVsrc { UVS_P16 = 0, UVS_PCN = 1, UVS_SP = 2 };

struct UDesc {
  uint32_t q0x, q0y, q0z, q0w, q1x, q1y, q1z, q1w;
};

struct UDescB {  // builder
  uint32_t xsel = PS_ZERO, psel = PS_ZERO, easel = PS_ZERO, k16 = 0, flags = 0;
  uint32_t keep = 0xF0, comp = 0, set = 0, xr = 0;
  uint32_t len = 1, cnt = 1, ct = 1, d8pos = 0, unit = UU_PASS, lop = 0, lsel = 0, rsel = 0, rkind = 0, tsel = 0,
           nw = 0;
  uint32_t cmask = 0, cval = 0, d16 = 0, vsrc = 0, spd = 0;

  __host__ __device__ constexpr void cyc(int c) { cnt = ct = (uint32_t)(c / 4); }
  __host__ __device__ constexpr void cyc2(int taken, int not_taken) {
    ct = (uint32_t)(taken / 4);
    cnt = (uint32_t)(not_taken / 4);
  }
  __host__ __device__ constexpr void x_reg(int r) { xsel = ps_reg(r); }
  __host__ __device__ constexpr void dst8(int r) {
    flags |= UF_D8 | ((r & 4) ? UF_D8_HI : 0u);
    d8pos = (uint32_t)((~r & 3) << 3);
  }
  __host__ __device__ constexpr void pair(int p) {  // 0 BC, 1 DE, 2 HL, 3 SP
    if (p == 3) flags |= UF_P_SP;
    else psel = p == 0 ? PS_BC : p == 1 ? PS_DE : PS_HL;
  }
  __host__ __device__ constexpr void ea_pair(int p) {  // 0 BC, 1 DE, 2 HL
    easel = p == 0 ? PS_BC : p == 1 ? PS_DE : PS_HL;
  }
  __host__ __device__ constexpr void read_hl() {
    ea_pair(2);
    flags |= UF_RD1 | UF_X_MEM;
  }
  __host__ __device__ constexpr void cond(int cc) {  // 0 NZ, 1 Z, 2 NC, 3 C
    cmask = (cc & 2) ? 0x10u : 0x80u;
    cval = (cc & 1) ? cmask : 0u;
  }
  __host__ __device__ constexpr void push_at_sp() { flags |= UF_EA_SP | UF_EA_DEC; nw = 2; spd = 1; }
  // flags: keep / computed / set / xor masks
  __host__ __device__ constexpr void fl(uint32_t k, uint32_t c, uint32_t s, uint32_t x = 0) {
    keep = k; comp = c; set = s; xr = x;
  }
  // ADD ADC SUB SBC AND XOR OR CP of A and x (alu.py); writes A except CP
  __host__ __device__ constexpr void alu(int kind) {
    if (kind < 4 || kind == 7) {
      unit = UU_ADD; lsel = ULS_A; rsel = URS_X;
      if (kind == 2 || kind == 3 || kind == 7) flags |= UF_SUB;
      if (kind == 1 || kind == 3) flags |= UF_CIN;
      fl(0, 0xF0, 0);
    } else {
      unit = UU_LOGIC; lop = kind == 4 ? UL_AND : kind == 5 ? UL_XOR : UL_OR;
      fl(0, 0x80, kind == 4 ? 0x20 : 0);
    }
    if (kind != 7) dst8(7);
  }
  // rotate / shift / swap kind of x (bitops.py): RLC RRC RL RR SLA SRA SWAP SRL
  __host__ __device__ constexpr void rot(int kind) {
    unit = UU_ROT;
    rkind = (uint32_t)kind;
  }

  __host__ __device__ constexpr UDesc build() const {
    UDesc d{};
    d.q0x = xsel | (psel << 16);
    d.q0y = easel | (k16 << 16);
    d.q0z = flags;
    d.q0w = keep | (comp << 8) | (set << 16) | (xr << 24);
    d.q1x = (len << UV_LEN) | (cnt << UV_CYC_NT) | (ct << UV_CYC_T) | (d8pos << UV_D8POS) | (unit << UV_UNIT) |
            (lop << UV_LOP) | (lsel << UV_LSEL) | (rsel << UV_RSEL) | (tsel << UV_TSEL) | (nw << UV_NW);
    d.q1y = cmask | (cval << 8) | (d16 << UY_D16) | (vsrc << UY_VSRC) | (spd << UY_SPD);
    d.q1z = rkind << 9;  // rotate-table row of the kind (see make_rot_table)
    return d;
  }
};

// Descriptor of key = opcode, or 256 + second byte for CB-prefixed opcodes.
// Opcode fields: x = op >> 6, y = (op >> 3) & 7, z = op & 7, p = y >> 1.
__host__ __device__ constexpr UDesc make_udesc(int key) {
  UDescB b{};
  if (key >= 256) {  // CB-prefixed (bitops.py)
    const int cb = key - 256, cz = cb & 7, cy = (cb >> 3) & 7, grp = cb >> 6;
    b.len = 2;
    if (cz == 6) b.read_hl(); else b.x_reg(cz);
    if (grp == 0) { b.rot(cy); b.fl(0, cy == 6 ? 0x80 : 0x90, 0); }
    else {
      b.unit = UU_LOGIC;
      b.flags |= UF_LX | UF_QK;
      if (grp == 1) { b.lop = UL_AND; b.k16 = 1u << cy; b.fl(0x10, 0x80, 0x20); }        // BIT
      else if (grp == 2) { b.lop = UL_AND; b.k16 = (~(1u << cy)) & 0xFF; }             // RES
      else { b.lop = UL_OR; b.k16 = 1u << cy; }                                          // SET
    }
    if (grp == 1) b.cyc(cz == 6 ? 12 : 8);
    else if (cz == 6) { b.nw = 1; b.cyc(16); }
    else { b.dst8(cz); b.cyc(8); }
    return b.build();
  }
  const int op = key, x = op >> 6, y = (op >> 3) & 7, z = op & 7, p = y >> 1;
  // traps: STOP and the unimplemented opcodes (misc.py:42-56)
  if (op == 0x10 || op == 0xD3 || op == 0xDB || op == 0xDD || op == 0xE3 || op == 0xE4 || op == 0xEB ||
      op == 0xEC || op == 0xED || op == 0xF4 || op == 0xFC || op == 0xFD || op == 0xCB) {
    b.flags |= UF_SPECIAL;
    b.cyc(0);
    return b.build();
  }
  if (x == 1) {
    if (op == 0x76) { b.flags |= UF_SPECIAL; return b.build(); }  // HALT
    if (z == 6) { b.read_hl(); b.dst8(y); b.cyc(8); }             // LD r,(HL)
    else if (y == 6) { b.ea_pair(2); b.x_reg(z); b.nw = 1; b.cyc(8); }  // LD (HL),r
    else { b.x_reg(z); b.dst8(y); }                               // LD r,r'
    return b.build();
  }
  if (x == 2) {  // ALU A,r / A,(HL)
    if (z == 6) { b.read_hl(); b.cyc(8); } else b.x_reg(z);
    b.alu(y);
    return b.build();
  }
  if (x == 0) {
    switch (z) {
      case 0:
        if (op == 0x00) return b.build();                          // NOP
        if (op == 0x08) {                                           // LD (a16),SP
          b.flags |= UF_EA_IMM16 | UF_LOFIRST; b.nw = 2; b.vsrc = UVS_SP; b.len = 3; b.cyc(20);
          return b.build();
        }
        b.len = 2; b.tsel = UT_JR;                                  // JR e8 / JR cc,e8
        if (op == 0x18) b.cyc(12);
        else { b.cond(y - 4); b.cyc2(12, 8); }
        return b.build();
      case 1:
        if (y & 1) {                                                // ADD HL,rr
          b.ea_pair(2); b.lsel = ULS_EA; b.rsel = URS_P16; b.pair(p);
          b.unit = UU_ADD; b.flags |= UF_WIDE; b.fl(0x80, 0x70, 0); b.d16 = UD_HL; b.cyc(8);
        } else {                                                    // LD rr,d16
          b.flags |= UF_EA_IMM16; b.lsel = ULS_EA; b.rsel = URS_K;
          b.d16 = p == 0 ? UD_BC : p == 1 ? UD_DE : p == 2 ? UD_HL : UD_SP;
          b.len = 3; b.cyc(12);
        }
        return b.build();
      case 2: {                                                     // LD (rr),A / LD A,(rr), HL+/-
        b.ea_pair(p < 2 ? p : 2);
        if (y & 1) { b.flags |= UF_RD1 | UF_X_MEM; b.dst8(7); }
        else { b.x_reg(7); b.nw = 1; }
        if (p >= 2) { b.lsel = ULS_EA; b.rsel = URS_K; b.k16 = p == 2 ? 1 : 0xFFFF; b.d16 = UD_HL; }
        b.cyc(8);
        return b.build();
      }
      case 3:                                                       // INC rr / DEC rr
        b.pair(p); b.lsel = ULS_P16; b.rsel = URS_K; b.k16 = (y & 1) ? 0xFFFF : 1;
        b.d16 = p == 0 ? UD_BC : p == 1 ? UD_DE : p == 2 ? UD_HL : UD_SP;
        b.cyc(8);
        return b.build();
      case 4: case 5:                                               // INC / DEC r or (HL)
        if (y == 6) { b.read_hl(); b.nw = 1; b.cyc(12); } else { b.x_reg(y); b.dst8(y); }
        b.unit = UU_ADD; b.lsel = ULS_X; b.rsel = URS_K; b.k16 = 1;
        if (z == 5) b.flags |= UF_SUB;
        b.fl(0x10, 0xE0, 0);
        return b.build();
      case 6:                                                       // LD r,d8 / LD (HL),d8
        b.flags |= UF_X_IMM; b.len = 2;
        if (y == 6) { b.ea_pair(2); b.nw = 1; b.cyc(12); } else { b.dst8(y); b.cyc(8); }
        return b.build();
      default:                                                      // z == 7
        if (y < 4) { b.x_reg(7); b.rot(y); b.dst8(7); b.fl(0, 0x10, 0); }   // RLCA RRCA RLA RRA
        else if (y == 4) b.flags |= UF_SPECIAL;                           // DAA
        else if (y == 5) {                                                // CPL
          b.unit = UU_LOGIC; b.lop = UL_XOR; b.flags |= UF_QK; b.k16 = 0xFF; b.dst8(7); b.fl(0x90, 0, 0x60);
        } else if (y == 6) b.fl(0x80, 0, 0x10);                           // SCF
        else b.fl(0x90, 0, 0, 0x10);                                      // CCF
        return b.build();
    }
  }
  // x == 3
  switch (op) {
    case 0xC0: case 0xC8: case 0xD0: case 0xD8: case 0xC9: case 0xD9:   // RET cc / RET / RETI
      b.flags |= UF_EA_SP | UF_RD1 | UF_RD2; b.tsel = UT_V16; b.spd = 2;
      if (op == 0xC9 || op == 0xD9) b.cyc(16); else { b.cond(y); b.cyc2(20, 8); }
      if (op == 0xD9) b.flags |= UF_SPECIAL;
      return b.build();
    case 0xC1: case 0xD1: case 0xE1: case 0xF1:                         // POP
      b.flags |= UF_EA_SP | UF_RD1 | UF_RD2 | UF_R16_POP; b.spd = 2;
      b.d16 = p == 0 ? UD_BC : p == 1 ? UD_DE : p == 2 ? UD_HL : UD_AF;
      b.cyc(12);
      return b.build();
    case 0xC2: case 0xCA: case 0xD2: case 0xDA: case 0xC3:              // JP cc / JP
      b.tsel = UT_IMM16; b.len = 3;
      if (op == 0xC3) b.cyc(16); else { b.cond(y); b.cyc2(16, 12); }
      return b.build();
    case 0xE9: b.ea_pair(2); b.tsel = UT_EA; return b.build();           // JP (HL)
    case 0xC4: case 0xCC: case 0xD4: case 0xDC: case 0xCD:              // CALL cc / CALL
      b.push_at_sp(); b.vsrc = UVS_PCN; b.tsel = UT_IMM16; b.len = 3;
      if (op == 0xCD) b.cyc(24); else { b.cond(y); b.cyc2(24, 12); }
      return b.build();
    case 0xC5: case 0xD5: case 0xE5: case 0xF5:                         // PUSH
      b.push_at_sp(); b.vsrc = UVS_P16;
      if (p == 3) { b.psel = PS_AHI; b.flags |= UF_P_AF; } else b.pair(p);
      b.cyc(16);
      return b.build();
    case 0xE0: b.flags |= UF_EA_IMM8 | UF_EA_FF; b.x_reg(7); b.nw = 1; b.len = 2; b.cyc(12); return b.build();
    case 0xE2: b.easel = PS_C; b.flags |= UF_EA_FF; b.x_reg(7); b.nw = 1; b.cyc(8); return b.build();
    case 0xEA: b.flags |= UF_EA_IMM16; b.x_reg(7); b.nw = 1; b.len = 3; b.cyc(16); return b.build();
    case 0xF0:
      b.flags |= UF_EA_IMM8 | UF_EA_FF | UF_RD1 | UF_X_MEM; b.dst8(7); b.len = 2; b.cyc(12);
      return b.build();
    case 0xF2: b.easel = PS_C; b.flags |= UF_EA_FF | UF_RD1 | UF_X_MEM; b.dst8(7); b.cyc(8); return b.build();
    case 0xFA:
      b.flags |= UF_EA_IMM16 | UF_RD1 | UF_X_MEM; b.dst8(7); b.len = 3; b.cyc(16);
      return b.build();
    case 0xE8: case 0xF8:                                               // ADD SP,e8 / LD HL,SP+e8
      b.pair(3); b.lsel = ULS_P16; b.rsel = URS_E8; b.fl(0, 0x30, 0);
      b.unit = UU_ADD;  // flags from the adder's low-byte taps; Z and N cleared
      b.d16 = op == 0xE8 ? UD_SP : UD_HL; b.len = 2; b.cyc(op == 0xE8 ? 16 : 12);
      return b.build();
    case 0xF9: b.ea_pair(2); b.lsel = ULS_EA; b.rsel = URS_K; b.d16 = UD_SP; b.cyc(8); return b.build();  // LD SP,HL
    case 0xF3: case 0xFB: b.flags |= UF_SPECIAL; return b.build();      // DI / EI
    default: break;
  }
  if (z == 6) { b.flags |= UF_X_IMM; b.len = 2; b.cyc(8); b.alu(y); return b.build(); }  // ALU A,d8
  // RST (z == 7)
  b.push_at_sp(); b.vsrc = UVS_PCN; b.tsel = UT_K; b.k16 = (uint32_t)(op & 0x38); b.cyc(16);
  return b.build();
}

// Rotate / shift / swap unit as a table (bitops.py): entry (kind << 9) |
// (carry << 8) | x holds the result byte and the carry out (bit 8) of kind
// RLC RRC RL RR SLA SRA SWAP SRL (0..7) applied to x with carry in `carry`
// (SWAP's carry out is 0).
__host__ __device__ constexpr uint32_t rot_entry(int kind, int c, int x) {
  int r = 0, co = 0;
  switch (kind) {
    case 0: co = x >> 7; r = ((x << 1) & 0xFF) | co; break;
    case 1: co = x & 1; r = (x >> 1) | (co << 7); break;
    case 2: co = x >> 7; r = ((x << 1) & 0xFF) | c; break;
    case 3: co = x & 1; r = (x >> 1) | (c << 7); break;
    case 4: co = x >> 7; r = (x << 1) & 0xFF; break;
    case 5: co = x & 1; r = (x >> 1) | (x & 0x80); break;
    case 6: co = 0; r = ((x & 0xF) << 4) | (x >> 4); break;
    default: co = x & 1; r = x >> 1; break;
  }
  return (uint32_t)r | ((uint32_t)co << 8);
}
constexpr int ROT_ENTRIES = 8 * 2 * 256;
struct RotTable {
  uint16_t v[ROT_ENTRIES];
};
__host__ __device__ constexpr RotTable make_rot_table() {
  RotTable t{};
  for (int k = 0; k < ROT_ENTRIES; k++) t.v[k] = (uint16_t)rot_entry(k >> 9, (k >> 8) & 1, k & 0xFF);
  return t;
}

constexpr int UDESC_KEYS = 512;
struct UDescTable {
  UDesc d[UDESC_KEYS];
};
__host__ __device__ constexpr UDescTable make_udesc_table() {
  UDescTable t{};
  for (int k = 0; k < UDESC_KEYS; k++) t.d[k] = make_udesc(k);
  return t;
}

}  // namespace gbx
