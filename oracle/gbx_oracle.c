/*
 * gbx_oracle.c - CPU restatement of the reference emulator step.
 *
 * TEST INFRASTRUCTURE ONLY: this is the checker the CUDA library is compared
 * against and the timed CPU baseline. The product never links or calls it.
 *
 * It restates, function by function, the Warp kernel of bkase/gbxcule:
 *   src/gbxcule/kernels/cpu_step_builder.py   (skeleton, :128-1782)
 *   src/gbxcule/kernels/cpu_templates/ (the instruction templates)
 *   src/gbxcule/kernels/cpu_step.py:130-341    (template map, stage bodies)
 *   src/gbxcule/kernels/ppu_render_downsampled.py:27-234 (snapshot renderer)
 *   src/gbxcule/kernels/reset_mask.py, src/gbxcule/core/reset_cache.py
 * with the reference's data layout: a flat u8[65536] address space per env,
 * env-major, and one array per scalar field. Quirks are kept on purpose; the
 * parity target is the reference kernel, not DMG hardware.
 *
 * Parity pin: tests/golden/ holds digests produced by running the reference's
 * own source (ref_harness.py) on the same ROMs, boot stub and action traces.
 */
#include <stdint.h>
#include <string.h>

#define MEM_SIZE 65536
#define CYCLES_PER_FRAME 70224
#define CYCLES_PER_SCANLINE 456
#define LINES_PER_FRAME 154
#define SCREEN_H 144
#define ROM_LIMIT 0x8000
#define CART_RAM_START 0xA000
#define CART_RAM_END 0xC000
#define ROM_BANK_SIZE 0x4000
#define RAM_BANK_SIZE 0x2000
#define BOOTROM_SIZE 0x100
#define CS_STRIDE 20
#define RTC_CPS 4194304
#define SERIAL_MAX 1024
#define OBS_DIM 32

enum { CS_MBC_KIND, CS_RAM_ENABLE, CS_ROM_BANK_LO, CS_ROM_BANK_HI, CS_RAM_BANK,
       CS_BANK_MODE, CS_BOOTROM, CS_RTC_SELECT, CS_RTC_LATCH, CS_RTC_S, CS_RTC_M,
       CS_RTC_H, CS_RTC_DL, CS_RTC_DH, CS_RTC_LAST, CS_RTC_LS, CS_RTC_LM, CS_RTC_LH,
       CS_RTC_LDL, CS_RTC_LDH };
enum { MBC_ROM_ONLY = 0, MBC_MBC1 = 1, MBC_MBC3 = 2 };
enum { STAGE_EMULATE = 0, STAGE_OBS = 1, STAGE_REWARD = 2, STAGE_FULL = 3 };

typedef struct {
    /* shared, read-only */
    const uint8_t *rom;
    const uint8_t *bootrom;
    int32_t rom_bank_count, rom_bank_mask, ram_bank_count;
    /* per env */
    uint8_t *mem;
    uint8_t *cart_ram;
    int32_t *cart_state;
    int32_t *pc, *sp, *a, *b, *c, *d, *e, *h, *l, *f;
    int64_t *instr_count, *cycle_count;
    int32_t *cycle_in_frame, *trap_flag, *trap_pc, *trap_opcode, *trap_kind;
    const int32_t *actions;
    uint8_t *joyp_select;
    uint8_t *serial_buf;
    int32_t *serial_len;
    uint8_t *serial_overflow;
    int32_t *ime, *ime_delay, *halted, *div_counter, *timer_prev_in;
    int32_t *tima_reload_pending, *tima_reload_delay;
    int32_t *ppu_scanline_cycle, *ppu_ly, *ppu_window_line;
    uint8_t *ppu_stat_prev;
    uint8_t *latch[9]; /* lcdc scx scy bgp wx wy win_line obp0 obp1, u8[144] */
    float *reward_out, *obs_out;
    int32_t stage, num_envs;
    /* optional (NULL = off): per env, bytes of RAM/IO (0x8000-0xFFFF, cart RAM
     * included) read or written by the emulated instructions, OAM DMA copies
     * counted as 160 read + 160 written. ROM and boot-ROM reads are not
     * counted (instruction fetch and ROM data: shared, read-only). Measures
     * the M_ops + D_dma terms of the step's algorithmic bytes; no effect on
     * the emulation. */
    int64_t *ram_ops;
} gbxo_ctx;

typedef struct {
    const gbxo_ctx *x;
    int32_t i;
    int64_t base;
    int32_t frames_done, release_after_frames;
} envref;

/* cpu_step_builder.py:196-247 */
static int action_dpad_mask(int action) {
    switch (action) { case 4: return 4; case 5: return 8; case 6: return 2; case 7: return 1; }
    return 0;
}
static int action_button_mask(int action) {
    switch (action) { case 1: return 1; case 2: return 2; case 3: return 8; }
    return 0;
}
static int joyp_read(int action, int frame_idx, int release_after_frames, int joyp_sel) {
    int sel = joyp_sel & 0x30;
    int pressed = frame_idx < release_after_frames;
    int dpad = 0, btn = 0;
    if (pressed) { dpad = action_dpad_mask(action); btn = action_button_mask(action); }
    int directional = 0x0F & ~dpad, standard = 0x0F & ~btn;
    int p14 = (sel >> 4) & 1, p15 = (sel >> 5) & 1;
    int v = (sel | 0xCF) & 0xFF;
    if (p14 && p15) v = 0x0F;
    else if (!p14 && !p15) { }
    else if (!p14) v &= directional;
    else v &= standard;
    return v | 0xC0;
}

/* :249-372 */
static int timer_div_bit(int tac) {
    switch (tac & 3) { case 0: return 9; case 1: return 3; case 2: return 5; }
    return 7;
}
static int timer_in(int div, int tac) {
    if ((tac & 4) == 0) return 0;
    return (div >> timer_div_bit(tac)) & 1;
}
static void tima_inc(const envref *r) {
    uint8_t *m = r->x->mem + r->base;
    int tima = m[0xFF05];
    m[0xFF05] = (uint8_t)((tima + 1) & 0xFF);
    if (tima == 0xFF) { r->x->tima_reload_pending[r->i] = 1; r->x->tima_reload_delay[r->i] = 4; }
}
static void tima_reload_now(const envref *r) {
    uint8_t *m = r->x->mem + r->base;
    m[0xFF05] = m[0xFF06];
    m[0xFF0F] |= 0x04;
    r->x->tima_reload_pending[r->i] = 0;
    r->x->tima_reload_delay[r->i] = 0;
}
static void timer_tick(const envref *r, int cycles) {
    if (cycles <= 0) return;
    const gbxo_ctx *x = r->x;
    int i = r->i;
    uint8_t *m = x->mem + r->base;
    int remaining = cycles;
    int div = x->div_counter[i] & 0xFFFF;
    while (remaining > 0) {
        if (x->tima_reload_pending[i] && x->tima_reload_delay[i] <= 0) tima_reload_now(r);
        int tac = m[0xFF07] & 7;
        int dt = remaining;
        if (x->tima_reload_pending[i]) { int rd = x->tima_reload_delay[i]; if (rd < dt) dt = rd; }
        int do_edge = 0;
        if (tac & 4) {
            int bit = timer_div_bit(tac);
            int period = 1 << (bit + 1);
            int edge_dt = period - (div & (period - 1));
            if (edge_dt < dt) dt = edge_dt;
            if (dt == edge_dt) do_edge = 1;
        }
        div = (div + dt) & 0xFFFF;
        if (x->tima_reload_pending[i]) x->tima_reload_delay[i] -= dt;
        remaining -= dt;
        if (do_edge) tima_inc(r);
        if (x->tima_reload_pending[i] && x->tima_reload_delay[i] <= 0) tima_reload_now(r);
    }
    x->div_counter[i] = div;
    m[0xFF04] = (uint8_t)((div >> 8) & 0xFF);
    x->timer_prev_in[i] = timer_in(div, m[0xFF07] & 7);
}

/* :375-419 */
static void rtc_tick(const envref *r, int cycles) {
    if (cycles <= 0) return;
    int32_t *cs = r->x->cart_state + (int64_t)r->i * CS_STRIDE;
    if (cs[CS_MBC_KIND] != MBC_MBC3) return;
    int days_high = cs[CS_RTC_DH];
    if (days_high & 0x40) return;
    int sub = cs[CS_RTC_LAST];
    if (sub < 0) sub = 0;
    sub += cycles;
    int sec = cs[CS_RTC_S] & 0xFF, minute = cs[CS_RTC_M] & 0x3F, hour = cs[CS_RTC_H] & 0x1F;
    int day = ((days_high & 1) << 8) | (cs[CS_RTC_DL] & 0xFF);
    while (sub >= RTC_CPS) {
        sub -= RTC_CPS;
        if (++sec >= 60) {
            sec = 0;
            if (++minute >= 60) {
                minute = 0;
                if (++hour >= 24) {
                    hour = 0;
                    if (++day >= 512) { day %= 512; days_high |= 0x80; }
                }
            }
        }
    }
    cs[CS_RTC_S] = sec; cs[CS_RTC_M] = minute; cs[CS_RTC_H] = hour;
    cs[CS_RTC_DL] = day & 0xFF;
    cs[CS_RTC_DH] = (days_high & 0xC0) | ((day >> 8) & 1);
    cs[CS_RTC_LAST] = sub;
}

/* :422-492 */
static void ppu_update_stat(uint8_t *m, int ly, int mode) {
    int coincidence = (ly == m[0xFF45]);
    m[0xFF41] = (uint8_t)((m[0xFF41] & 0xF8) | (coincidence << 2) | mode);
}
static void ppu_update_stat_irq(const envref *r, uint8_t *m, int ly, int mode) {
    int coincidence = (ly == m[0xFF45]);
    int keep = m[0xFF41] & 0xF8;
    m[0xFF41] = (uint8_t)(keep | (coincidence << 2) | mode);
    int en0 = (keep >> 3) & 1, en1 = (keep >> 4) & 1, en2 = (keep >> 5) & 1, enl = (keep >> 6) & 1;
    int c0 = mode == 0, c1 = mode == 1, c2 = mode == 2, cl = coincidence;
    int prev = r->x->ppu_stat_prev[r->i] & 0x0F;
    int edge = 0;
    if (en0 && !(prev & 1) && c0) edge = 1;
    else if (en1 && !((prev >> 1) & 1) && c1) edge = 1;
    else if (en2 && !((prev >> 2) & 1) && c2) edge = 1;
    else if (enl && !((prev >> 3) & 1) && cl) edge = 1;
    if (edge) m[0xFF0F] |= 0x02;
    r->x->ppu_stat_prev[r->i] = (uint8_t)(c0 | (c1 << 1) | (c2 << 2) | (cl << 3));
}
/* :495-525 */
static void latch_env0(const envref *r, uint8_t *m, int ly, int win_line) {
    if (r->i != 0) return;
    if (ly < 0 || ly >= SCREEN_H) return;
    uint8_t *const *L = r->x->latch;
    L[0][ly] = m[0xFF40]; L[1][ly] = m[0xFF43]; L[2][ly] = m[0xFF42]; L[3][ly] = m[0xFF47];
    L[4][ly] = m[0xFF4B]; L[5][ly] = m[0xFF4A]; L[6][ly] = (uint8_t)(win_line & 0xFF);
    L[7][ly] = m[0xFF48]; L[8][ly] = m[0xFF49];
}

/* PPU advance block, written out three times in the skeleton
 * (:1403-1500 after an instruction, :988-1082 in HALT, :1601-1704 after an
 * interrupt service). Returns the LCDC value it read. */
static int ppu_advance(const envref *r, int cycles, int *scan, int *ly, int *wl) {
    uint8_t *m = r->x->mem + r->base;
    int lcdc = m[0xFF40];
    if ((lcdc & 0x80) == 0) {
        *scan = 0; *ly = 0; *wl = 0;
        m[0xFF44] = 0;
        ppu_update_stat(m, 0, 0);
        r->x->ppu_stat_prev[r->i] = 0;
        return lcdc;
    }
    int total = *scan + cycles;
    int lines = total / CYCLES_PER_SCANLINE;
    *scan = total - lines * CYCLES_PER_SCANLINE;
    if (lines == 0 && *scan == 0) latch_env0(r, m, *ly, *wl);
    while (lines > 0) {
        int prev_ly = *ly;
        if (prev_ly < SCREEN_H && (lcdc & 0x20) && prev_ly >= m[0xFF4A]) (*wl)++;
        *ly = (*ly + 1) % LINES_PER_FRAME;
        if (*ly == 0) *wl = 0;
        m[0xFF44] = (uint8_t)*ly;
        ppu_update_stat_irq(r, m, *ly, *ly >= SCREEN_H ? 1 : 0);
        if (prev_ly == 143 && *ly == 144) m[0xFF0F] |= 0x01;
        if (*ly < SCREEN_H) latch_env0(r, m, *ly, *wl);
        lines--;
    }
    int mode = *ly >= SCREEN_H ? 1 : (*scan < 80 ? 2 : (*scan < 250 ? 3 : 0));
    ppu_update_stat(m, *ly, mode);
    int cl = (*ly == m[0xFF45]);
    r->x->ppu_stat_prev[r->i] = (uint8_t)((mode == 0) | ((mode == 1) << 1) | ((mode == 2) << 2) | (cl << 3));
    return lcdc;
}

/* :527-536 */
static int clamp_bank(int bank, int count, int mask) {
    if (count <= 0) return 0;
    if (mask >= 0) return bank & mask;
    return bank % count;
}

/* :539-657 */
static int read8(const envref *r, int addr) {
    const gbxo_ctx *x = r->x;
    int a16 = addr & 0xFFFF;
    if (a16 >= 0xE000 && a16 < 0xFE00) a16 -= 0x2000;
    if (x->ram_ops && a16 >= ROM_LIMIT) x->ram_ops[r->i]++;
    const int32_t *cs = x->cart_state + (int64_t)r->i * CS_STRIDE;
    if (a16 < BOOTROM_SIZE && cs[CS_BOOTROM] != 0) return x->bootrom[a16];
    if (a16 < ROM_LIMIT) {
        int mbc = cs[CS_MBC_KIND];
        int lo_raw = cs[CS_ROM_BANK_LO], lo = lo_raw & 0x1F, hi = cs[CS_ROM_BANK_HI] & 3;
        int mode = cs[CS_BANK_MODE] & 1;
        int bank = 0;
        if (a16 < 0x4000) {
            if (mbc == MBC_MBC1 && mode) bank = (hi & 3) << 5;
        } else if (mbc == MBC_ROM_ONLY) {
            bank = 1;
        } else if (mbc == MBC_MBC1) {
            bank = (hi << 5) | lo;
            if (bank == 0) bank = 1;
        } else {
            bank = lo_raw & 0x7F;
            if (bank == 0) bank = 1;
        }
        bank = clamp_bank(bank, x->rom_bank_count, x->rom_bank_mask);
        int idx = bank * ROM_BANK_SIZE + (a16 < 0x4000 ? a16 : a16 - 0x4000);
        if (idx < x->rom_bank_count * ROM_BANK_SIZE) return x->rom[idx];
        return 0xFF;
    }
    const uint8_t *m = x->mem + r->base;
    if (a16 == 0xFF00) return m[0xFF00];
    if (a16 >= CART_RAM_START && a16 < CART_RAM_END) {
        if (x->ram_bank_count <= 0) return 0xFF;
        if (cs[CS_RAM_ENABLE] == 0) return 0xFF;
        int mbc = cs[CS_MBC_KIND];
        if (mbc == MBC_MBC3) {
            int sel = cs[CS_RTC_SELECT] & 0x0F;
            int latched = cs[CS_RTC_LATCH] != 0;
            if (sel >= 0x08 && sel <= 0x0C)
                return (latched ? cs[CS_RTC_LS + (sel - 8)] : cs[CS_RTC_S + (sel - 8)]) & 0xFF;
        }
        int rb = 0;
        if (mbc == MBC_MBC1) { if (cs[CS_BANK_MODE] & 1) rb = cs[CS_RAM_BANK] & 3; }
        else if (mbc == MBC_MBC3) rb = cs[CS_RAM_BANK] & 3;
        rb = clamp_bank(rb, x->ram_bank_count, -1);
        int env_bytes = x->ram_bank_count * RAM_BANK_SIZE;
        if (env_bytes <= 0) return 0xFF;
        int off = rb * RAM_BANK_SIZE + (a16 - CART_RAM_START);
        if (off >= env_bytes) return 0xFF;
        return x->cart_ram[(int64_t)r->i * env_bytes + off];
    }
    return m[a16];
}

/* :660-873 */
static void write8(const envref *r, int addr, int val) {
    const gbxo_ctx *x = r->x;
    int i = r->i;
    int a16 = addr & 0xFFFF;
    if (a16 >= 0xE000 && a16 < 0xFE00) a16 -= 0x2000;
    uint8_t v8 = (uint8_t)val;
    uint8_t *m = x->mem + r->base;
    int32_t *cs = x->cart_state + (int64_t)i * CS_STRIDE;
    if (x->ram_ops && a16 >= ROM_LIMIT) x->ram_ops[i] += a16 == 0xFF46 ? 321 : 1;
    switch (a16) {
    case 0xFF00: {
        int sel = v8 & 0x30;
        x->joyp_select[i] = (uint8_t)sel;
        m[0xFF00] = (uint8_t)joyp_read(x->actions[i], r->frames_done, r->release_after_frames, sel);
        return;
    }
    case 0xFF0F: m[a16] = v8 & 0x1F; return;
    case 0xFF01: m[a16] = v8; return;
    case 0xFF02:
        m[a16] = v8;
        if ((val & 0x80) && (val & 0x01)) {
            int sb = m[0xFF01];
            int idx = x->serial_len[i];
            if (idx < SERIAL_MAX) { x->serial_buf[(int64_t)i * SERIAL_MAX + idx] = (uint8_t)sb; x->serial_len[i] = idx + 1; }
            else x->serial_overflow[i] = 1;
            m[a16] = (uint8_t)(val & 0x7F);
            m[0xFF0F] |= 0x08;
        }
        return;
    case 0xFF50: if (val != 0) cs[CS_BOOTROM] = 0; return;
    case 0xFF04: {
        int tac = m[0xFF07] & 7;
        int pre = timer_in(x->div_counter[i] & 0xFFFF, tac);
        m[a16] = 0;
        x->div_counter[i] = 0;
        int post = timer_in(0, tac);
        x->timer_prev_in[i] = post;
        if (pre && !post) tima_inc(r);
        return;
    }
    case 0xFF05: case 0xFF06: m[a16] = v8; return;
    case 0xFF07: {
        int div = x->div_counter[i] & 0xFFFF;
        int pre = timer_in(div, m[0xFF07] & 7);
        int tac_new = val & 7;
        m[a16] = (uint8_t)tac_new;
        int post = timer_in(div, tac_new);
        x->timer_prev_in[i] = post;
        if (pre && !post) tima_inc(r);
        return;
    }
    case 0xFF46: {
        m[a16] = v8;
        int src = (val & 0xFF) << 8;
        for (int o = 0; o < 160; o++) m[0xFE00 + o] = m[(src + o) & 0xFFFF];
        return;
    }
    case 0xFFFF: m[a16] = v8 & 0x1F; return;
    default: break;
    }
    if (a16 >= CART_RAM_START && a16 < CART_RAM_END) {
        if (x->ram_bank_count <= 0) return;
        if (cs[CS_RAM_ENABLE] == 0) return;
        int mbc = cs[CS_MBC_KIND];
        if (mbc == MBC_MBC3) {
            int sel = cs[CS_RTC_SELECT] & 0x0F;
            if (sel >= 0x08 && sel <= 0x0C) { cs[CS_RTC_S + (sel - 8)] = val & 0xFF; return; }
        }
        int rb = 0;
        if (mbc == MBC_MBC1) { if (cs[CS_BANK_MODE] & 1) rb = cs[CS_RAM_BANK] & 3; }
        else if (mbc == MBC_MBC3) rb = cs[CS_RAM_BANK] & 3;
        rb = clamp_bank(rb, x->ram_bank_count, -1);
        int env_bytes = x->ram_bank_count * RAM_BANK_SIZE;
        if (env_bytes <= 0) return;
        int off = rb * RAM_BANK_SIZE + (a16 - CART_RAM_START);
        if (off >= env_bytes) return;
        x->cart_ram[(int64_t)i * env_bytes + off] = v8;
        return;
    }
    if (a16 < ROM_LIMIT) {
        int mbc = cs[CS_MBC_KIND];
        if (mbc == MBC_MBC1) {
            if (a16 < 0x2000) cs[CS_RAM_ENABLE] = (val & 0x0F) == 0x0A;
            else if (a16 < 0x4000) { int bk = val & 0x1F; if (!bk) bk = 1; cs[CS_ROM_BANK_LO] = bk; }
            else if (a16 < 0x6000) { int bk = val & 3; cs[CS_ROM_BANK_HI] = bk; cs[CS_RAM_BANK] = bk; }
            else cs[CS_BANK_MODE] = val & 1;
        } else if (mbc == MBC_MBC3) {
            if (a16 < 0x2000) cs[CS_RAM_ENABLE] = (val & 0x0F) == 0x0A;
            else if (a16 < 0x4000) { int bk = val & 0x7F; if (!bk) bk = 1; cs[CS_ROM_BANK_LO] = bk; }
            else if (a16 < 0x6000) { int sel = val & 0x0F; cs[CS_RTC_SELECT] = sel; if (sel <= 3) cs[CS_RAM_BANK] = sel; }
            else {
                if (val == 0) cs[CS_RTC_LATCH] = 0;
                else if (val == 1 && cs[CS_RTC_LATCH] == 0) {
                    for (int k = 0; k < 5; k++) cs[CS_RTC_LS + k] = cs[CS_RTC_S + k];
                    cs[CS_RTC_LATCH] = 1;
                }
            }
        }
        return;
    }
    m[a16] = v8;
}

/* make_flags (:190-192) */
#define FLAGS(z, n, hh, cc) (((z) << 7) | ((n) << 6) | ((hh) << 5) | ((cc) << 4))
static int sign8(int v) { return v >= 128 ? v - 256 : v; }

typedef struct {
    int pc, sp, a, b, c, d, e, h, l, f;
    int trap, trap_pc, trap_op, trap_kind;
} cpu_t;

static int *r8(cpu_t *s, int code) {
    switch (code) { case 0: return &s->b; case 1: return &s->c; case 2: return &s->d; case 3: return &s->e;
                    case 4: return &s->h; case 5: return &s->l; default: return &s->a; }
}
static int *hi16(cpu_t *s, int rr) { return rr == 0 ? &s->b : rr == 1 ? &s->d : &s->h; }
static int *lo16(cpu_t *s, int rr) { return rr == 0 ? &s->c : rr == 1 ? &s->e : &s->l; }
#define HL(s) ((((s)->h << 8) | (s)->l) & 0xFFFF)

/* 8-bit ALU templates (alu.py:59-70, 285-297, 299-456, 458-640, 642-744) */
static void alu8(cpu_t *s, int kind, int v) {
    int a = s->a, res, z, hf, cf, carry;
    switch (kind) {
    case 0: /* ADD */
        res = a + v; z = (res & 0xFF) == 0;
        hf = ((a & 0xF) + (v & 0xF)) > 0xF; cf = res > 0xFF;
        s->a = res & 0xFF; s->f = FLAGS(z, 0, hf, cf); break;
    case 1: /* ADC */
        carry = (s->f >> 4) & 1; res = a + v + carry; z = (res & 0xFF) == 0;
        hf = ((a & 0xF) + (v & 0xF) + carry) > 0xF; cf = res > 0xFF;
        s->a = res & 0xFF; s->f = FLAGS(z, 0, hf, cf); break;
    case 2: /* SUB */
        res = a - v; z = (res & 0xFF) == 0;
        hf = ((a & 0xF) - (v & 0xF)) < 0; cf = a < v;
        s->a = res & 0xFF; s->f = FLAGS(z, 1, hf, cf); break;
    case 3: /* SBC */
        carry = (s->f >> 4) & 1; res = a - v - carry; z = (res & 0xFF) == 0;
        hf = ((a & 0xF) - ((v & 0xF) + carry)) < 0; cf = a < (v + carry);
        s->a = res & 0xFF; s->f = FLAGS(z, 1, hf, cf); break;
    case 4: /* AND */
        s->a = (a & v) & 0xFF; s->f = FLAGS(s->a == 0, 0, 1, 0); break;
    case 5: /* XOR */
        s->a = (a ^ v) & 0xFF; s->f = FLAGS(s->a == 0, 0, 0, 0); break;
    case 6: /* OR */
        s->a = (a | v) & 0xFF; s->f = FLAGS(s->a == 0, 0, 0, 0); break;
    default: /* CP */
        res = a - v; z = (res & 0xFF) == 0;
        hf = ((a & 0xF) - (v & 0xF)) < 0; cf = a < v;
        s->f = FLAGS(z, 1, hf, cf); break;
    }
}

/* CB rotate/shift family (bitops.py:46-570); returns the new value */
static int cb_shift(cpu_t *s, int kind, int v) {
    int cf, res, oc = (s->f >> 4) & 1;
    switch (kind) {
    case 0: cf = (v >> 7) & 1; res = ((v << 1) & 0xFF) | cf; break;          /* RLC */
    case 1: cf = v & 1; res = ((v >> 1) & 0xFF) | (cf << 7); break;          /* RRC */
    case 2: cf = (v >> 7) & 1; res = ((v << 1) & 0xFF) | oc; break;          /* RL */
    case 3: cf = v & 1; res = ((v >> 1) & 0xFF) | (oc << 7); break;          /* RR */
    case 4: cf = (v >> 7) & 1; res = (v << 1) & 0xFF; break;                 /* SLA */
    case 5: cf = v & 1; res = ((v >> 1) & 0x7F) | (v & 0x80); break;         /* SRA */
    case 6: cf = 0; res = ((v & 0x0F) << 4) | ((v & 0xF0) >> 4); break;      /* SWAP */
    default: cf = v & 1; res = (v >> 1) & 0x7F; break;                       /* SRL */
    }
    s->f = FLAGS(res == 0, 0, 0, cf);
    return res;
}

static int push16(const envref *r, cpu_t *s, int val) {
    s->sp = (s->sp - 1) & 0xFFFF; write8(r, s->sp, (val >> 8) & 0xFF);
    s->sp = (s->sp - 1) & 0xFFFF; write8(r, s->sp, val & 0xFF);
    return 0;
}
static int pop16(const envref *r, cpu_t *s) {
    int lo = read8(r, s->sp); s->sp = (s->sp + 1) & 0xFFFF;
    int hi = read8(r, s->sp); s->sp = (s->sp + 1) & 0xFFFF;
    return ((hi << 8) | lo) & 0xFFFF;
}
static int cond_true(const cpu_t *s, int cc) {
    switch (cc & 3) {
    case 0: return ((s->f >> 7) & 1) == 0;
    case 1: return ((s->f >> 7) & 1) != 0;
    case 2: return ((s->f >> 4) & 1) == 0;
    default: return ((s->f >> 4) & 1) != 0;
    }
}

/* One unprefixed instruction; returns cycles. Template per opcode follows
 * core/isa_sm83.py's table and cpu_step.py:130-258. */
static int exec_op(const envref *r, cpu_t *s, int op) {
    const gbxo_ctx *x = r->x;
    int i = r->i;
    int pc = s->pc;
#define RD(ad) read8(r, (ad))
#define IMM8 RD((pc + 1) & 0xFFFF)
#define IMM16 ((RD((pc + 2) & 0xFFFF) << 8) | RD((pc + 1) & 0xFFFF))
    /* LD r,r' / LD r,(HL) / LD (HL),r (loads.py) */
    if (op >= 0x40 && op < 0x80 && op != 0x76) {
        int dst = (op >> 3) & 7, src = op & 7;
        if (src == 6) { *r8(s, dst) = RD(HL(s)); s->pc = (pc + 1) & 0xFFFF; return 8; }
        if (dst == 6) { write8(r, HL(s), *r8(s, src)); s->pc = (pc + 1) & 0xFFFF; return 8; }
        *r8(s, dst) = *r8(s, src) & 0xFF; s->pc = (pc + 1) & 0xFFFF; return 4;
    }
    if (op >= 0x80 && op < 0xC0) {
        int src = op & 7;
        if (src == 6) { alu8(s, (op >> 3) & 7, RD(HL(s))); s->pc = (pc + 1) & 0xFFFF; return 8; }
        alu8(s, (op >> 3) & 7, *r8(s, src)); s->pc = (pc + 1) & 0xFFFF; return 4;
    }
    switch (op) {
    case 0x00: s->pc = (pc + 1) & 0xFFFF; return 4;
    case 0x01: case 0x11: case 0x21: { int v = IMM16 & 0xFFFF, rr = op >> 4;
        *hi16(s, rr) = (v >> 8) & 0xFF; *lo16(s, rr) = v & 0xFF; s->pc = (pc + 3) & 0xFFFF; return 12; }
    case 0x31: s->sp = IMM16 & 0xFFFF; s->pc = (pc + 3) & 0xFFFF; return 12;
    case 0x02: write8(r, ((s->b << 8) | s->c) & 0xFFFF, s->a); s->pc = (pc + 1) & 0xFFFF; return 8;
    case 0x12: write8(r, ((s->d << 8) | s->e) & 0xFFFF, s->a); s->pc = (pc + 1) & 0xFFFF; return 8;
    case 0x0A: s->a = RD(((s->b << 8) | s->c) & 0xFFFF); s->pc = (pc + 1) & 0xFFFF; return 8;
    case 0x1A: s->a = RD(((s->d << 8) | s->e) & 0xFFFF); s->pc = (pc + 1) & 0xFFFF; return 8;
    case 0x22: case 0x32: { int hl = HL(s); write8(r, hl, s->a);
        hl = (op == 0x22 ? hl + 1 : hl - 1) & 0xFFFF; s->h = hl >> 8; s->l = hl & 0xFF;
        s->pc = (pc + 1) & 0xFFFF; return 8; }
    case 0x2A: case 0x3A: { int hl = HL(s); s->a = RD(hl);
        hl = (op == 0x2A ? hl + 1 : hl - 1) & 0xFFFF; s->h = hl >> 8; s->l = hl & 0xFF;
        s->pc = (pc + 1) & 0xFFFF; return 8; }
    case 0x03: case 0x13: case 0x23: case 0x0B: case 0x1B: case 0x2B: {
        int rr = (op >> 4) & 3, v = ((*hi16(s, rr) << 8) | *lo16(s, rr)) & 0xFFFF;
        v = ((op & 8) ? v - 1 : v + 1) & 0xFFFF;
        *hi16(s, rr) = (v >> 8) & 0xFF; *lo16(s, rr) = v & 0xFF; s->pc = (pc + 1) & 0xFFFF; return 8; }
    case 0x33: s->sp = (s->sp + 1) & 0xFFFF; s->pc = (pc + 1) & 0xFFFF; return 8;
    case 0x3B: s->sp = (s->sp - 1) & 0xFFFF; s->pc = (pc + 1) & 0xFFFF; return 8;
    case 0x04: case 0x0C: case 0x14: case 0x1C: case 0x24: case 0x2C: case 0x3C: {
        int *p = r8(s, (op >> 3) & 7), old = *p; *p = (*p + 1) & 0xFF;
        s->f = FLAGS(*p == 0, 0, (old & 0xF) == 0xF, (s->f >> 4) & 1); s->pc = (pc + 1) & 0xFFFF; return 4; }
    case 0x05: case 0x0D: case 0x15: case 0x1D: case 0x25: case 0x2D: case 0x3D: {
        int *p = r8(s, (op >> 3) & 7), old = *p; *p = (*p - 1) & 0xFF;
        s->f = FLAGS(*p == 0, 1, (old & 0xF) == 0, (s->f >> 4) & 1); s->pc = (pc + 1) & 0xFFFF; return 4; }
    case 0x34: case 0x35: { int hl = HL(s), v = RD(hl), old = v;
        v = (op == 0x34 ? v + 1 : v - 1) & 0xFF; write8(r, hl, v);
        if (op == 0x34) s->f = FLAGS(v == 0, 0, (old & 0xF) == 0xF, (s->f >> 4) & 1);
        else s->f = FLAGS(v == 0, 1, (old & 0xF) == 0, (s->f >> 4) & 1);
        s->pc = (pc + 1) & 0xFFFF; return 12; }
    case 0x06: case 0x0E: case 0x16: case 0x1E: case 0x26: case 0x2E: case 0x3E:
        *r8(s, (op >> 3) & 7) = IMM8; s->pc = (pc + 2) & 0xFFFF; return 8;
    case 0x36: { int v = IMM8; write8(r, HL(s), v); s->pc = (pc + 2) & 0xFFFF; return 12; }
    case 0x07: { int cf = (s->a >> 7) & 1; s->a = ((s->a << 1) & 0xFF) | cf; s->f = FLAGS(0, 0, 0, cf); s->pc = (pc + 1) & 0xFFFF; return 4; }
    case 0x0F: { int cf = s->a & 1; s->a = ((s->a >> 1) & 0xFF) | (cf << 7); s->f = FLAGS(0, 0, 0, cf); s->pc = (pc + 1) & 0xFFFF; return 4; }
    case 0x17: { int oc = (s->f >> 4) & 1, cf = (s->a >> 7) & 1; s->a = ((s->a << 1) & 0xFF) | oc; s->f = FLAGS(0, 0, 0, cf); s->pc = (pc + 1) & 0xFFFF; return 4; }
    case 0x1F: { int oc = (s->f >> 4) & 1, cf = s->a & 1; s->a = ((s->a >> 1) & 0xFF) | (oc << 7); s->f = FLAGS(0, 0, 0, cf); s->pc = (pc + 1) & 0xFFFF; return 4; }
    case 0x08: { int ad = IMM16 & 0xFFFF; write8(r, ad, s->sp & 0xFF); write8(r, (ad + 1) & 0xFFFF, (s->sp >> 8) & 0xFF);
        s->pc = (pc + 3) & 0xFFFF; return 20; }
    case 0x09: case 0x19: case 0x29: case 0x39: {
        int hl = HL(s), rr = op == 0x39 ? s->sp : (((*hi16(s, (op >> 4) & 3)) << 8) | *lo16(s, (op >> 4) & 3)) & 0xFFFF;
        int sum = hl + rr;
        int hf = ((hl & 0x0FFF) + (rr & 0x0FFF)) > 0x0FFF, cf = sum > 0xFFFF;
        s->h = (sum >> 8) & 0xFF; s->l = sum & 0xFF;
        s->f = FLAGS((s->f >> 7) & 1, 0, hf, cf); s->pc = (pc + 1) & 0xFFFF; return 8; }
    case 0x18: { int off = sign8(IMM8); s->pc = (pc + 2 + off) & 0xFFFF; return 12; }
    case 0x20: case 0x28: case 0x30: case 0x38: { int off = sign8(IMM8);
        if (cond_true(s, (op >> 3) & 3)) { s->pc = (pc + 2 + off) & 0xFFFF; return 12; }
        s->pc = (pc + 2) & 0xFFFF; return 8; }
    case 0x27: { /* DAA alu.py:897-922 */
        int av = s->a & 0xFF, n = (s->f >> 6) & 1, hf = (s->f >> 5) & 1, cf = (s->f >> 4) & 1;
        int adj = 0, carry = cf;
        if (!n) {
            if (hf || (av & 0x0F) > 9) adj |= 0x06;
            if (cf || av > 0x99) { adj |= 0x60; carry = 1; }
            av = (av + adj) & 0xFF;
        } else {
            if (hf) adj |= 0x06;
            if (cf) adj |= 0x60;
            av = (av - adj) & 0xFF;
        }
        s->f = FLAGS(av == 0, n, 0, carry); s->a = av; s->pc = (pc + 1) & 0xFFFF; return 4; }
    case 0x2F: s->a ^= 0xFF; s->f = FLAGS((s->f >> 7) & 1, 1, 1, (s->f >> 4) & 1); s->pc = (pc + 1) & 0xFFFF; return 4;
    case 0x37: s->f = FLAGS((s->f >> 7) & 1, 0, 0, 1); s->pc = (pc + 1) & 0xFFFF; return 4;
    case 0x3F: s->f = FLAGS((s->f >> 7) & 1, 0, 0, ((s->f >> 4) & 1) ? 0 : 1); s->pc = (pc + 1) & 0xFFFF; return 4;
    case 0x76: x->halted[i] = 1; s->pc = (pc + 1) & 0xFFFF; return 4;
    case 0xF3: x->ime[i] = 0; x->ime_delay[i] = 0; s->pc = (pc + 1) & 0xFFFF; return 4;
    case 0xFB: x->ime[i] = 1; x->ime_delay[i] = 0; s->pc = (pc + 1) & 0xFFFF; return 4;
    case 0xC6: case 0xCE: case 0xD6: case 0xDE: case 0xE6: case 0xEE: case 0xF6: case 0xFE:
        alu8(s, (op >> 3) & 7, IMM8); s->pc = (pc + 2) & 0xFFFF; return 8;
    case 0xC3: s->pc = IMM16 & 0xFFFF; return 16;
    case 0xC2: case 0xCA: case 0xD2: case 0xDA: { int ad = IMM16 & 0xFFFF;
        if (cond_true(s, (op >> 3) & 3)) { s->pc = ad; return 16; }
        s->pc = (pc + 3) & 0xFFFF; return 12; }
    case 0xE9: s->pc = HL(s); return 4;
    case 0xCD: { int ad = IMM16 & 0xFFFF; push16(r, s, (pc + 3) & 0xFFFF); s->pc = ad; return 24; }
    case 0xC4: case 0xCC: case 0xD4: case 0xDC:
        if (cond_true(s, (op >> 3) & 3)) { int ad = IMM16 & 0xFFFF; push16(r, s, (pc + 3) & 0xFFFF); s->pc = ad; return 24; }
        s->pc = (pc + 3) & 0xFFFF; return 12;
    case 0xC9: s->pc = pop16(r, s); return 16;
    case 0xD9: s->pc = pop16(r, s); x->ime[i] = 1; x->ime_delay[i] = 0; return 16;
    case 0xC0: case 0xC8: case 0xD0: case 0xD8:
        if (cond_true(s, (op >> 3) & 3)) { s->pc = pop16(r, s); return 20; }
        s->pc = (pc + 1) & 0xFFFF; return 8;
    case 0xC7: case 0xCF: case 0xD7: case 0xDF: case 0xE7: case 0xEF: case 0xF7: case 0xFF:
        push16(r, s, (pc + 1) & 0xFFFF); s->pc = op & 0x38; return 16;
    case 0xC1: case 0xD1: case 0xE1: { int rr = (op >> 4) & 3, v = pop16(r, s);
        *hi16(s, rr) = (v >> 8) & 0xFF; *lo16(s, rr) = v & 0xFF; s->pc = (pc + 1) & 0xFFFF; return 12; }
    case 0xF1: { int v = pop16(r, s); s->a = (v >> 8) & 0xFF; s->f = v & 0xF0; s->pc = (pc + 1) & 0xFFFF; return 12; }
    case 0xC5: case 0xD5: case 0xE5: { int rr = (op >> 4) & 3;
        push16(r, s, ((*hi16(s, rr) & 0xFF) << 8) | (*lo16(s, rr) & 0xFF)); s->pc = (pc + 1) & 0xFFFF; return 16; }
    case 0xF5: push16(r, s, ((s->a & 0xFF) << 8) | (s->f & 0xF0)); s->pc = (pc + 1) & 0xFFFF; return 16;
    case 0xE0: { int ad = (0xFF00 | IMM8) & 0xFFFF; write8(r, ad, s->a); s->pc = (pc + 2) & 0xFFFF; return 12; }
    case 0xF0: { int ad = (0xFF00 | IMM8) & 0xFFFF; s->a = RD(ad); s->pc = (pc + 2) & 0xFFFF; return 12; }
    case 0xE2: write8(r, (0xFF00 | s->c) & 0xFFFF, s->a); s->pc = (pc + 1) & 0xFFFF; return 8;
    case 0xF2: s->a = RD((0xFF00 | s->c) & 0xFFFF); s->pc = (pc + 1) & 0xFFFF; return 8;
    case 0xEA: write8(r, IMM16 & 0xFFFF, s->a); s->pc = (pc + 3) & 0xFFFF; return 16;
    case 0xFA: s->a = RD(IMM16 & 0xFFFF); s->pc = (pc + 3) & 0xFFFF; return 16;
    case 0xE8: case 0xF8: { int off = IMM8, os = sign8(off), ou = off & 0xFF;
        int hf = ((s->sp & 0xF) + (ou & 0xF)) > 0xF, cf = ((s->sp & 0xFF) + ou) > 0xFF;
        int res = (s->sp + os) & 0xFFFF;
        if (op == 0xE8) { s->sp = res; s->pc = (pc + 2) & 0xFFFF; s->f = FLAGS(0, 0, hf, cf); return 16; }
        s->h = (res >> 8) & 0xFF; s->l = res & 0xFF; s->f = FLAGS(0, 0, hf, cf); s->pc = (pc + 2) & 0xFFFF; return 12; }
    case 0xF9: s->sp = HL(s); s->pc = (pc + 1) & 0xFFFF; return 8;
    default:
        /* misc.py:42-56 template_trap_unprefixed (STOP and the illegal set) */
        if (s->trap == 0) { s->trap = 1; s->trap_pc = pc & 0xFFFF; s->trap_op = op & 0xFF; s->trap_kind = 1; }
        return 0;
    }
#undef RD
#undef IMM8
#undef IMM16
}

/* CB-prefixed instruction; pc already advanced by 2 (:1339-1360). */
static int exec_cb(const envref *r, cpu_t *s, int cb) {
    int reg = cb & 7, grp = cb >> 6, y = (cb >> 3) & 7;
    int is_hl = reg == 6;
    int hl = HL(s);
    int v = is_hl ? read8(r, hl) : *r8(s, reg);
    switch (grp) {
    case 0: v = cb_shift(s, y, v); break;
    case 1: /* BIT (bitops.py:573-590) */
        s->f = FLAGS(((v >> y) & 1) == 0, 0, 1, (s->f >> 4) & 1);
        return is_hl ? 12 : 8;
    case 2: v = v & (0xFF ^ (1 << y)); break;
    default: v = v | (1 << y); break;
    }
    if (is_hl) { write8(r, hl, v); return 16; }
    *r8(s, reg) = v;
    return 8;
}

/* Interrupt service (:1502-1604 / :1086-1183): clears IME and the IF bit,
 * pushes PC through write8, jumps to the vector. */
static void service(const envref *r, cpu_t *s, int pending) {
    uint8_t *m = r->x->mem + r->base;
    int vector, bit;
    if (pending & 1) { vector = 0x40; bit = 1; }
    else if (pending & 2) { vector = 0x48; bit = 2; }
    else if (pending & 4) { vector = 0x50; bit = 4; }
    else if (pending & 8) { vector = 0x58; bit = 8; }
    else { vector = 0x60; bit = 0x10; }
    r->x->ime[r->i] = 0;
    m[0xFF0F] &= (uint8_t)(0xFF ^ bit);
    int ret = s->pc & 0xFFFF;
    s->sp = (s->sp - 1) & 0xFFFF; write8(r, s->sp, (ret >> 8) & 0xFF);
    s->sp = (s->sp - 1) & 0xFFFF; write8(r, s->sp, ret & 0xFF);
    s->pc = vector;
}

/* post_step.py:11-102 */
static void post_step(const gbxo_ctx *x, int i, const cpu_t *s) {
    const uint8_t *m = x->mem + (int64_t)i * MEM_SIZE;
    if (x->stage == STAGE_OBS || x->stage == STAGE_FULL) {
        float *o = x->obs_out + (int64_t)i * OBS_DIM;
        o[0] = (float)(s->pc & 0xFFFF) / 65535.0f;
        o[1] = (float)(s->sp & 0xFFFF) / 65535.0f;
        o[2] = (float)(s->a & 0xFF) / 255.0f;
        o[3] = (float)(s->f & 0xFF) / 255.0f;
        o[4] = (float)(s->b & 0xFF) / 255.0f;
        o[5] = (float)(s->c & 0xFF) / 255.0f;
        o[6] = (float)(s->d & 0xFF) / 255.0f;
        o[7] = (float)(s->e & 0xFF) / 255.0f;
        o[8] = (float)(s->h & 0xFF) / 255.0f;
        o[9] = (float)(s->l & 0xFF) / 255.0f;
        for (int k = 0; k < 16; k++) o[10 + k] = (float)m[0xC000 + k] / 255.0f;
        int m0 = m[0xC000], m1 = m[0xC001], m2 = m[0xC002], m3 = m[0xC003];
        int m4 = m[0xC004], m5 = m[0xC005], m6 = m[0xC006], m7 = m[0xC007];
        o[26] = (float)((m0 ^ m1) & 0xFF) / 255.0f;
        o[27] = (float)((m2 + m3 * 5) & 0xFF) / 255.0f;
        o[28] = (float)((m4 ^ (s->a & 0xFF)) & 0xFF) / 255.0f;
        o[29] = (float)((m5 + (s->b & 0xFF)) & 0xFF) / 255.0f;
        o[30] = (float)((m6 ^ (s->c & 0xFF)) & 0xFF) / 255.0f;
        o[31] = (float)((m7 + (s->d & 0xFF)) & 0xFF) / 255.0f;
    }
    if (x->stage == STAGE_REWARD || x->stage == STAGE_FULL) {
        int mix = (m[0xC000] + m[0xC001] * 3) & 0xFF;
        x->reward_out[i] = (float)((s->a ^ mix) & 0xFF) / 255.0f;
    }
}

/* Debug traps of the reference kernel (cpu_step.py:85-105 reads them from
 * GBXCULE_TRAP_PC, GBXCULE_TRAP_RST38, GBXCULE_MAX_INSTR, GBXCULE_WATCH_ADDR;
 * 0 = off). */
typedef struct {
    int32_t trap_pc, trap_rst38, watch_addr, pad;
    int64_t max_instr;
} gbxo_debug;

static void set_trap(cpu_t *s, int pc, int op, int kind) {
    if (s->trap == 0) { s->trap = 1; s->trap_pc = pc & 0xFFFF; s->trap_op = op & 0xFF; s->trap_kind = kind; }
}

/* The per-env body of cpu_step (:876-1781). */
static void step_env(const gbxo_ctx *x, int i, int frames_to_run, int release_after_frames,
                     const gbxo_debug *dbg) {
    envref rr = { x, i, (int64_t)i * MEM_SIZE, 0, release_after_frames };
    envref *r = &rr;
    uint8_t *m = x->mem + rr.base;
    cpu_t s;
    s.pc = x->pc[i] & 0xFFFF; s.sp = x->sp[i] & 0xFFFF;
    s.a = x->a[i] & 0xFF; s.b = x->b[i] & 0xFF; s.c = x->c[i] & 0xFF; s.d = x->d[i] & 0xFF;
    s.e = x->e[i] & 0xFF; s.h = x->h[i] & 0xFF; s.l = x->l[i] & 0xFF; s.f = x->f[i] & 0xF0;
    s.trap = x->trap_flag[i]; s.trap_pc = x->trap_pc[i]; s.trap_op = x->trap_opcode[i]; s.trap_kind = x->trap_kind[i];
    int64_t instr = x->instr_count[i], cyc = x->cycle_count[i];
    int cycle_frame = x->cycle_in_frame[i];
    int scan = x->ppu_scanline_cycle[i], ly = x->ppu_ly[i], wl = x->ppu_window_line[i];
    const int64_t instr_start = instr;                                   /* :946-951 */
    const int watch_val = dbg->watch_addr ? m[dbg->watch_addr & 0xFFFF] : 0;

    while (rr.frames_done < frames_to_run) {
        if (s.trap) break;
        int lcdc_prev = m[0xFF40] & 0x80;
        if (x->halted[i]) {
            int cycles = 4;
            timer_tick(r, cycles);
            int lcdc = ppu_advance(r, cycles, &scan, &ly, &wl);
            int pending = m[0xFFFF] & m[0xFF0F] & 0x1F;
            int svc = 0;
            if (pending) {
                x->halted[i] = 0;
                if (x->ime[i]) {
                    service(r, &s, pending);
                    svc = 20;
                    timer_tick(r, svc);
                } else {
                    s.pc = (s.pc + 1) & 0xFFFF; /* :1181-1183 */
                }
            }
            if (svc) lcdc = ppu_advance(r, svc, &scan, &ly, &wl);
            int total = cycles + svc;
            rtc_tick(r, total);
            cyc += total;
            cycle_frame += total;
            if (lcdc_prev && !(lcdc & 0x80)) {
                cycle_frame = 0;
                rr.frames_done++;
                continue;
            }
            while (cycle_frame >= CYCLES_PER_FRAME) {
                cycle_frame -= CYCLES_PER_FRAME;
                rr.frames_done++;
                if (rr.frames_done >= frames_to_run) break;
            }
            continue;
        }
        int pc_before = s.pc;
        int opcode = read8(r, s.pc);
        /* :1320-1338 checks before execution */
        if (dbg->trap_pc && s.pc == dbg->trap_pc) { set_trap(&s, s.pc, opcode, 5); break; }
        if (dbg->trap_rst38 && opcode == 0xFF && s.pc != 0x0038) { set_trap(&s, s.pc, opcode, 3); break; }
        int cycles;
        if (opcode == 0xCB) {
            int cb = read8(r, (s.pc + 1) & 0xFFFF);
            s.pc = (s.pc + 2) & 0xFFFF;
            cycles = exec_cb(r, &s, cb);
        } else {
            cycles = exec_op(r, &s, opcode);
        }
        /* :1362-1393 checks after execution */
        if (dbg->trap_rst38 && s.pc >= 0xFE00) { set_trap(&s, pc_before, opcode, 4); break; }
        if (s.trap) break;
        s.f &= 0xF0;
        instr++;
        if (dbg->max_instr > 0 && instr - instr_start >= dbg->max_instr) { set_trap(&s, s.pc, opcode, 6); break; }
        if (dbg->watch_addr && m[dbg->watch_addr & 0xFFFF] != watch_val) { set_trap(&s, pc_before, opcode, 7); break; }
        timer_tick(r, cycles);
        if (x->ime_delay[i]) { x->ime[i] = 1; x->ime_delay[i] = 0; }
        int lcdc = ppu_advance(r, cycles, &scan, &ly, &wl);
        int pending = m[0xFFFF] & m[0xFF0F] & 0x1F;
        int svc = 0;
        if (pending) {
            if (x->halted[i]) x->halted[i] = 0;
            if (x->ime[i]) {
                service(r, &s, pending);
                svc = 20;
                timer_tick(r, svc);
                lcdc = ppu_advance(r, svc, &scan, &ly, &wl);
            }
        }
        int total = cycles + svc;
        rtc_tick(r, total);
        cyc += total;
        cycle_frame += total;
        if (lcdc_prev && !(lcdc & 0x80)) {
            int tail = total;
            if (opcode == 0xE0) {
                int imm = read8(r, (pc_before + 1) & 0xFFFF);
                if ((imm & 0xFF) == 0x40 && cycles >= 4) tail = total - 4;
            }
            cycle_frame = tail;
            rr.frames_done++;
            continue;
        } else if (!lcdc_prev && (lcdc & 0x80)) {
            scan = 0; ly = 0; wl = 0;
            m[0xFF44] = 0;
            ppu_update_stat(m, 0, 2);
            int cl = m[0xFF45] == 0;
            x->ppu_stat_prev[i] = (uint8_t)((1 << 2) | (cl << 3));
            cycle_frame = 0;
            rr.frames_done++;
            continue;
        } else {
            while (cycle_frame >= CYCLES_PER_FRAME) {
                cycle_frame -= CYCLES_PER_FRAME;
                rr.frames_done++;
                if (rr.frames_done >= frames_to_run) break;
            }
        }
    }
    post_step(x, i, &s);
    x->pc[i] = s.pc & 0xFFFF; x->sp[i] = s.sp & 0xFFFF;
    x->a[i] = s.a & 0xFF; x->b[i] = s.b & 0xFF; x->c[i] = s.c & 0xFF; x->d[i] = s.d & 0xFF;
    x->e[i] = s.e & 0xFF; x->h[i] = s.h & 0xFF; x->l[i] = s.l & 0xFF; x->f[i] = s.f & 0xF0;
    x->instr_count[i] = instr; x->cycle_count[i] = cyc; x->cycle_in_frame[i] = cycle_frame;
    x->ppu_scanline_cycle[i] = scan; x->ppu_ly[i] = ly; x->ppu_window_line[i] = wl;
    x->trap_flag[i] = s.trap; x->trap_pc[i] = s.trap_pc; x->trap_opcode[i] = s.trap_op; x->trap_kind[i] = s.trap_kind;
}

/* ------------------------------------------------------------------------ */
/* Exported entry points (ctypes)                                            */
/* ------------------------------------------------------------------------ */

void gbxo_step_debug(const gbxo_ctx *x, int32_t env_lo, int32_t env_hi, int32_t frames_to_run,
                     int32_t release_after_frames, int32_t nthreads, const gbxo_debug *dbg) {
#ifdef _OPENMP
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int i = env_lo; i < env_hi; i++) step_env(x, i, frames_to_run, release_after_frames, dbg);
    (void)nthreads;
}

void gbxo_step(const gbxo_ctx *x, int32_t env_lo, int32_t env_hi, int32_t frames_to_run,
               int32_t release_after_frames, int32_t nthreads) {
    const gbxo_debug off = {0, 0, 0, 0, 0};
    gbxo_step_debug(x, env_lo, env_hi, frames_to_run, release_after_frames, nthreads, &off);
}

/* kernels/ppu_step.py:11-176: env 0's 160x144 frame from the per-line
 * register latches (window row = the latched window line) and env 0's
 * current VRAM/OAM. latch: lcdc, scx, scy, bgp, wx, wy, win_line, obp0, obp1. */
void gbxo_render_bg_env0(const uint8_t *m, const uint8_t *const *latch, uint8_t *out) {
    for (int y = 0; y < SCREEN_H; y++) {
        const int lcdc = latch[0][y], scx = latch[1][y], scy = latch[2][y], bgp = latch[3][y];
        const int wx = latch[4][y], wy = latch[5][y], win_line = latch[6][y];
        const int obp0 = latch[7][y], obp1 = latch[8][y];
        for (int x = 0; x < 160; x++) {
            int shade = 0, bg_color = 0;
            if (lcdc & 0x01) {
                const int use_win = (lcdc & 0x20) && y >= wy && x >= wx - 7;
                int px, py, map;
                if (use_win) { px = x - (wx - 7); py = win_line; map = (lcdc & 0x40) ? 0x9C00 : 0x9800; }
                else { px = (x + scx) & 0xFF; py = (y + scy) & 0xFF; map = (lcdc & 0x08) ? 0x9C00 : 0x9800; }
                int tile_id = m[map + ((py & 0xFF) >> 3) * 32 + ((px & 0xFF) >> 3)];
                int ta = (lcdc & 0x10) ? 0x8000 + tile_id * 16 : 0x9000 + (tile_id >= 128 ? tile_id - 256 : tile_id) * 16;
                int row = py & 7;
                int lo = m[ta + row * 2], hi = m[ta + row * 2 + 1];
                int bit = 7 - (px & 7);
                bg_color = (((hi >> bit) & 1) << 1) | ((lo >> bit) & 1);
                shade = (bgp >> (bg_color * 2)) & 3;
            }
            if (lcdc & 0x02) {
                const int sh = (lcdc & 0x04) ? 16 : 8;
                int on_line = 0, found = 0, best_x = 0, best_color = 0, best_attr = 0;
                for (int k = 0; k < 40; k++) {
                    const int sy = m[0xFE00 + 4 * k], sx = m[0xFE00 + 4 * k + 1];
                    int tile = m[0xFE00 + 4 * k + 2];
                    const int attr = m[0xFE00 + 4 * k + 3];
                    if (sx == 0 || sy == 0 || sx >= 168 || sy >= 160) continue;
                    const int top = sy - 16, left = sx - 8;
                    if (y < top || y >= top + sh) continue;
                    if (on_line >= 10) continue;
                    on_line++;
                    if (x < left || x >= left + 8) continue;
                    int row = y - top;
                    if ((attr >> 6) & 1) row = sh - 1 - row;
                    if (sh == 16) { tile &= 0xFE; if (row >= 8) { tile++; row -= 8; } }
                    const int ta = 0x8000 + tile * 16;
                    const int lo = m[ta + row * 2], hi = m[ta + row * 2 + 1];
                    const int pxo = x - left;
                    const int bit = ((attr >> 5) & 1) ? pxo : 7 - pxo;
                    const int color = (((hi >> bit) & 1) << 1) | ((lo >> bit) & 1);
                    if (color == 0) continue;
                    if (!found || left < best_x) { found = 1; best_x = left; best_color = color; best_attr = attr; }
                }
                if (found && !(((best_attr >> 7) & 1) && bg_color != 0))
                    shade = ((((best_attr >> 4) & 1) ? obp1 : obp0) >> (best_color * 2)) & 3;
            }
            out[y * 160 + x] = (uint8_t)shade;
        }
    }
}

/* ppu_render_downsampled.py:27-179 */
static int sample_shade(const uint8_t *m, int x, int y) {
    int lcdc = m[0xFF40], scy = m[0xFF42], scx = m[0xFF43], bgp = m[0xFF47];
    int obp0 = m[0xFF48], obp1 = m[0xFF49], wy = m[0xFF4A], wx = m[0xFF4B];
    int shade = 0, bg_color = 0;
    if (lcdc & 1) {
        int use_win = (lcdc & 0x20) && y >= wy && x >= wx - 7;
        int px, py, map;
        if (use_win) { px = x - (wx - 7); py = y - wy; map = (lcdc & 0x40) ? 0x9C00 : 0x9800; }
        else { px = (x + scx) & 0xFF; py = (y + scy) & 0xFF; map = (lcdc & 0x08) ? 0x9C00 : 0x9800; }
        int tile_id = m[map + ((py & 0xFF) >> 3) * 32 + ((px & 0xFF) >> 3)];
        int tile_addr = (lcdc & 0x10) ? 0x8000 + tile_id * 16 : 0x9000 + (tile_id >= 128 ? tile_id - 256 : tile_id) * 16;
        int row = py & 7;
        int lo = m[tile_addr + row * 2], hi = m[tile_addr + row * 2 + 1];
        int bit = 7 - (px & 7);
        bg_color = (((hi >> bit) & 1) << 1) | ((lo >> bit) & 1);
        shade = (bgp >> (bg_color * 2)) & 3;
    }
    if (lcdc & 2) {
        int sh = (lcdc & 4) ? 16 : 8;
        int on_line = 0, found = 0, best_x = 0, best_oam = 0, best_color = 0, best_attr = 0;
        for (int s = 0; s < 40; s++) {
            int sy = m[0xFE00 + s * 4], sx = m[0xFE01 + s * 4], tile = m[0xFE02 + s * 4], attr = m[0xFE03 + s * 4];
            if (sx == 0 || sy == 0 || sx >= 168 || sy >= 160) continue;
            int top = sy - 16, left = sx - 8;
            if (y < top || y >= top + sh) continue;
            if (on_line >= 10) continue;
            on_line++;
            if (x < left || x >= left + 8) continue;
            int row = y - top;
            if ((attr >> 6) & 1) row = sh - 1 - row;
            if (sh == 16) { tile &= 0xFE; if (row >= 8) { tile++; row -= 8; } }
            int ta = 0x8000 + tile * 16;
            int lo = m[ta + row * 2], hi = m[ta + row * 2 + 1];
            int pxo = x - left;
            int bit = ((attr >> 5) & 1) ? pxo : 7 - pxo;
            int color = (((hi >> bit) & 1) << 1) | ((lo >> bit) & 1);
            if (color == 0) continue;
            if (!found) { found = 1; best_x = left; best_oam = s; best_color = color; best_attr = attr; }
            else if (left < best_x) { best_x = left; best_oam = s; best_color = color; best_attr = attr; }
            else if (left == best_x && s < best_oam) { best_oam = s; best_color = color; best_attr = attr; }
        }
        if (found) {
            int prio = (best_attr >> 7) & 1;
            if (!(prio && bg_color != 0)) {
                int pal = ((best_attr >> 4) & 1) ? obp1 : obp0;
                shade = (pal >> (best_color * 2)) & 3;
            }
        }
    }
    return shade;
}

/* :207-234 packed (72x20 bytes per env) and :182-204 unpacked (72x80). */
void gbxo_render(const uint8_t *mem, int32_t num_envs, uint8_t *out, int32_t packed, int32_t nthreads) {
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(nthreads > 0 ? nthreads : 1)
#endif
    for (int e = 0; e < num_envs; e++) {
        const uint8_t *m = mem + (int64_t)e * MEM_SIZE;
        for (int oy = 0; oy < 72; oy++) {
            if (packed) {
                for (int b = 0; b < 20; b++) {
                    int v = 0;
                    for (int k = 0; k < 4; k++) v |= (sample_shade(m, (b * 4 + k) * 2, oy * 2) & 3) << (2 * k);
                    out[(int64_t)e * 1440 + oy * 20 + b] = (uint8_t)v;
                }
            } else {
                for (int ox = 0; ox < 80; ox++) out[(int64_t)e * 5760 + oy * 80 + ox] = (uint8_t)sample_shade(m, ox * 2, oy * 2);
            }
        }
    }
    (void)nthreads;
}
