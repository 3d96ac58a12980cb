// qx_load.cu -- machine images <-> head states, on the device.
//
// The snapshot (ERV/chipformer/rv/core.py:1177-1270 with Executor2.load_init,
// ERV/chipformer/rv/tritonexec.py:246-258) writes a machine's registers, PC, counters, ROM (the
// pre-decoded words of ERV/chipformer/rv/ref.py:335-380), DROM, digit file and RAM into the
// rows of its head states; every other row is zero.  Here one warp builds one 512-byte row
// (lanes own 4 columns), so loading thousands of machines streams at HBM speed.  The readback
// inverts it for the registers, PC and RAM, and the checksum hashes the result (FNV-1a 64).
#include <cuda_runtime.h>

#include "qx_exec.cuh"

#define A_REF 16777216.0f
#define A_BIT 128.0f
#define ROM_BASE 0x40000u
#define ROM_WORDS 65536u
#define RAM_WORDS 8192u

// table indices in the plan's TABLES section
enum { T_PC = 0, T_COUNT = 1, T_J = 2, T_VCNT = 3, T_REGS = 4, T_QUO = 7, T_ROM = 11, T_DROM = 43,
       T_BN1 = 59, T_BN2 = 63, T_RAM = 67 };

namespace {

__device__ __forceinline__ int64_t sxd(uint32_t v, int bits) {
    uint64_t u = v & ((1ull << bits) - 1);
    return (u >> (bits - 1)) & 1 ? (int64_t)u - (int64_t)(1ull << bits) : (int64_t)u;
}

__device__ __forceinline__ uint32_t pk(uint32_t uop, uint32_t rd, uint32_t rs1, uint32_t rs2, uint32_t sp) {
    return (uop | (sp & 1) << 7) | (rd << 3 | (sp >> 1 & 7)) << 8 | (rs1 << 3 | (sp >> 4 & 7)) << 16 |
           (rs2 << 3 | (sp >> 7 & 7)) << 24;
}

// uop numbers of the pre-decoded ROM word (ref.py:55-68)
enum { U_ILLEGAL = 0, U_LUI = 1, U_AUIPC = 2, U_MISA = 3, U_ADDI = 4, U_SLLI = 10, U_SRLI = 11, U_SRAI = 12,
       U_ADD = 13, U_SUB = 14, U_SRA = 20, U_LB = 23, U_SB = 28, U_BEQ = 31, U_JAL = 37, U_JALR = 38,
       U_ECALL = 39, U_EBREAK = 40, U_FENCE = 41, U_MUL = 42, U_SH1ADD = 50, U_BMAC = 64, U_BPRD = 68 };

__device__ __forceinline__ bool in_rom(uint32_t t) { return t % 4 == 0 && t >= ROM_BASE && t < ROM_BASE + 4 * ROM_WORDS; }

// The pre-decoded ROM word of instruction w at pc (ref.py:344-380).
__device__ uint32_t rom_word(uint32_t w, uint32_t pc) {
    const uint32_t opc = w & 0x7F, rd = w >> 7 & 31, f3 = w >> 12 & 7, rs1 = w >> 15 & 31, rs2 = w >> 20 & 31,
                   f7 = w >> 25;
    const int64_t i_imm = sxd(w >> 20, 12);
    if (opc == 0x37 || opc == 0x17) {  // LUI / AUIPC: the upper 20 bits (AUIPC: of pc + imm)
        int64_t imm = sxd(w & 0xFFFFF000u, 32);
        uint32_t up = (uint32_t)(((opc == 0x37 ? imm : (int64_t)pc + imm) >> 12) & 0xFFFFF);
        return pk(opc == 0x37 ? U_LUI : U_AUIPC, rd, up & 31, up >> 5 & 31, up >> 10);
    }
    if (opc == 0x6F) {  // JAL: the target's word index and a bad-target flag
        int64_t j = sxd((w >> 31 & 1) << 20 | (w >> 12 & 0xFF) << 12 | (w >> 20 & 1) << 11 | (w >> 21 & 0x3FF) << 1, 21);
        uint32_t t = (uint32_t)(((int64_t)pc + j) & 0xFFFFFFFF);
        uint32_t wi = ((t - ROM_BASE) >> 2) & 0xFFFF;
        return pk(U_JAL, rd, wi & 31, wi >> 5 & 31, wi >> 10 | (uint32_t)!in_rom(t) << 6);
    }
    int32_t op = -1;  // I-type family: register + 12-bit immediate
    if (opc == 0x67 && f3 == 0) op = U_JALR;
    else if (opc == 0x03 && (f3 <= 2 || f3 == 4 || f3 == 5)) op = U_LB + (f3 <= 2 ? f3 : f3 - 1);  // LB LH LW LBU LHU
    else if (opc == 0x13) {
        if (f3 == 1 && f7 == 0) op = U_SLLI;
        else if (f3 == 5 && f7 == 0) op = U_SRLI;
        else if (f3 == 5 && f7 == 0x20) op = U_SRAI;
        else if (f3 != 1 && f3 != 5) {
            const int32_t I[8] = {U_ADDI, -1, 5, 6, 7, -1, 8, 9};  // ADDI SLTI SLTIU XORI ORI ANDI
            op = I[f3];
        }
    }
    if (op >= 0) {
        uint32_t imm = (op == U_SLLI || op == U_SRLI || op == U_SRAI) ? rs2 : (uint32_t)(i_imm & 0xFFF);
        return pk(op, rd, rs1, imm & 31, imm >> 5);
    }
    if (opc == 0x23 && f3 <= 2) {  // stores: RD slot = the data register
        uint32_t imm = (uint32_t)(sxd((w >> 25) << 5 | (w >> 7 & 31), 12) & 0xFFF);
        return pk(U_SB + f3, rs2, rs1, imm & 31, imm >> 5);
    }
    if (opc == 0x63 && f3 != 2 && f3 != 3) {  // branches: signed word offset and bad-target flag
        int64_t b = sxd((w >> 31 & 1) << 12 | (w >> 7 & 1) << 11 | (w >> 25 & 63) << 5 | (w >> 8 & 15) << 1, 13);
        uint32_t t = (uint32_t)(((int64_t)pc + b) & 0xFFFFFFFF);
        uint32_t off = (uint32_t)((b >> 2) & 0x7FF);
        const uint32_t B[8] = {31, 32, 0, 0, 33, 34, 35, 36};
        return pk(B[f3], off & 31, rs1, rs2, off >> 5 | (uint32_t)!in_rom(t) << 6);
    }
    if (opc == 0x33) {
        if (f7 == 0) {
            const uint32_t R[8] = {13, 15, 16, 17, 18, 19, 21, 22};  // ADD SLL SLT SLTU XOR SRL OR AND
            return pk(R[f3], rd, rs1, rs2, 0);
        }
        if (f7 == 0x20 && (f3 == 0 || f3 == 5)) return pk(f3 == 0 ? U_SUB : U_SRA, rd, rs1, rs2, 0);
        if (f7 == 1) return pk(U_MUL + f3, rd, rs1, rs2, 0);
        if (f7 == 0x10 && (f3 == 2 || f3 == 4 || f3 == 6)) return pk(U_SH1ADD + (f3 / 2 - 1), rd, rs1, rs2, 0);
    }
    if (opc == 0x0B && f3 < 5 && f7 == 0) {  // digit-file row ops: BMAC BMSB BLD BGET BSCAN
        const uint32_t C[5] = {64, 65, 66, 67, 69};
        return pk(C[f3], rd, rs1, rs2, 0);
    }
    if (opc == 0x2B && f3 == 0) {  // BPRD: k = imm[6:0], dD = rd & 7
        uint32_t imm = w >> 20 & 0x7F;
        return pk(U_BPRD, 0, 0, imm & 31, imm >> 5 | (rd & 7) << 7);
    }
    if (w == 0x00000073u) return pk(U_ECALL, 0, 17, 10, 0);
    if (opc == 0x73 && (f3 == 1 || f3 == 2 || f3 == 3 || f3 == 5 || f3 == 6 || f3 == 7)) {
        // CSR: pure reads (CSRRS/CSRRC/CSRRSI/CSRRCI with rs1 = 0) of the stubbed CSRs only
        bool pure = (f3 == 2 || f3 == 3 || f3 == 6 || f3 == 7) && rs1 == 0;
        uint32_t csr = w >> 20;
        bool zero = csr == 0xC00 || csr == 0xC01 || csr == 0xC02 || csr == 0xC80 || csr == 0xC81 ||
                    csr == 0xC82 || csr == 0xF14;
        if (!pure || (!zero && csr != 0x301)) return pk(U_ILLEGAL, 0, 0, 0, 0);
        return csr == 0x301 ? pk(U_MISA, rd, 0, 0, 0) : pk(U_LUI, rd, 0, 0, 0);
    }
    if (w == 0x00100073u) return pk(U_EBREAK, 0, 0, 0, 0);
    if (opc == 0x0F) return pk(U_FENCE, 0, 0, 0, 0);
    return pk(U_ILLEGAL, 0, 0, 0, 0);
}

__device__ __forceinline__ float *row_ptr(const QxDev &d, int t, int x, int r, int m) {
    const uint32_t hl = d.tables[2 * t], vh0 = d.tables[2 * t + 1];
    return d.S[hl] + (((size_t)m * d.V[hl] + vh0 + x) * QX_HD + r) * QX_HD;
}
// Whether table t lives in a shared sublayer (one copy per firmware image).
__device__ __forceinline__ bool shared_table(const QxDev &d, int t) { return d.shared_hl >> d.tables[2 * t] & 1u; }

#define QX_LOAD_TASKS 22636  // content rows a machine's load writes (the zero-row list follows)

// The state row load task `task` writes for machine m (the same map serves the loader and the
// coverage kernel that finds the rows no task writes)
__device__ __forceinline__ float *task_row(const QxDev &d, int task, int m) {
    if (task == 0) return row_ptr(d, T_PC, 0, 0, m);
    if (task < 7) return row_ptr(d, T_COUNT + (task - 1) / 2, 0, (task - 1) % 2, m);
    if (task < 100) return row_ptr(d, T_REGS + (task - 7) / 31, 0, 1 + (task - 7) % 31, m);
    if (task < 108) return row_ptr(d, T_QUO + (task - 100) / 2, (task - 100) % 2, 0, m);
    if (task < 12396) {
        const bool rom = task < 8300;
        const int k0 = rom ? task - 108 : task - 8300;
        return row_ptr(d, (rom ? T_ROM : T_DROM) + k0 / 256, (k0 / 128) % 2, k0 % 128, m);
    }
    if (task < 14444) {
        const int k0 = task - 12396;
        return row_ptr(d, (k0 / 1024 ? T_BN2 : T_BN1) + (k0 / 256) % 4, (k0 / 128) % 2, k0 % 128, m);
    }
    const uint32_t wi = (uint32_t)(task - 14444);
    return row_ptr(d, T_RAM + ((wi & 15) | (wi >> 12) << 4), wi >> 4 & 1, wi >> 5 & 127, m);
}

}  // namespace

// Marks, in cover[hl][row] (machine 0's rows), every state row a load task writes.
__global__ void qx_load_cover_kernel(const __grid_constant__ QxDev d, uint8_t *cover) {
    for (int task = blockIdx.x * blockDim.x + threadIdx.x; task < QX_LOAD_TASKS; task += gridDim.x * blockDim.x) {
        const float *row = task_row(d, task, 0);
        size_t base = 0;
        for (int hl = 0; hl < d.n_hl; hl++) {
            const size_t rows = (size_t)d.V[hl] * QX_HD;
            if (row >= d.S[hl] && row < d.S[hl] + rows * QX_HD) {
                cover[base + (size_t)(row - d.S[hl]) / QX_HD] = 1;
                break;
            }
            base += rows;
        }
    }
}

// Pre-decode every machine's ROM words in the pool, in place (zero words stay zero).
__global__ void qx_predecode_kernel(const QxImage *img, uint32_t *pool, int32_t n) {
    const int i = blockIdx.y;
    if (i >= n) return;
    const QxImage &im = img[i];  // read in place (a copy would live in local memory)
    for (uint32_t k = blockIdx.x * blockDim.x + threadIdx.x; k < im.rom_len; k += gridDim.x * blockDim.x) {
        uint32_t w = pool[im.rom_off + k];
        pool[im.rom_off + k] = w ? rom_word(w, ROM_BASE + 4 * k) : 0;
    }
}

// The small content rows, task [0, 108) of a machine: this lane's four columns and the row.
//   [0, 7) pc, count x2, j x2, vcnt x2   [7, 100) registers (3 ports x 31)   [100, 108) quotient
static __device__ __forceinline__ float *small_row(const QxDev &d, const QxImage &im, int task, int m, int lane,
                                                   float4 &out) {
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    float *row = nullptr;
    bool ballast = true;
    if (task < 7) {
        if (task == 0) {
            row = row_ptr(d, T_PC, 0, 0, m);
            for (int k = 0; k < 4; k++) {
                int c = lane * 4 + k;
                if (c >= 2 && c < 18) v[k] = (im.anchor >> (c - 2) & 1) ? A_BIT : 0.0f;
            }
        } else {
            const int t = T_COUNT + (task - 1) / 2, r = (task - 1) % 2;
            row = row_ptr(d, t, 0, r, m);
            if (r == 0) {
                ballast = false;
                if (lane == 0) v[2] = ldexpf(A_BIT, -(int)(t == T_COUNT ? im.n : 0));
            }
        }
    } else if (task < 100) {
        const int p = (task - 7) / 31, reg = 1 + (task - 7) % 31;
        row = row_ptr(d, T_REGS + p, 0, reg, m);
        for (int b = 0; b < 32; b++) {
            int c = d.reg_cols[b * 8];
            if (c >= 0 && c < QX_HD && (im.x[reg] >> b & 1) && c / 4 == lane) v[c % 4] = A_BIT;
        }
    } else {
        const int h = (task - 100) / 2, x = (task - 100) % 2;
        row = row_ptr(d, T_QUO + h, x, 0, m);
    }
    if (ballast && lane == 0) { v[0] = A_REF; v[1] = A_REF; }
    out = make_float4(v[0], v[1], v[2], v[3]);
    return row;
}

// Groups of four consecutive rows of one value head (tasks 108 + 4g .. 108 + 4g + 3 of the
// content rows, the RAM rows taken in row order):
//   [0, 2048) ROM   [2048, 3072) DROM   [3072, 3584) digit file   [3584, 5632) RAM
#define QX_LOAD_GROUPS 5632
#define QX_LOAD_SMALL 108

static __device__ __forceinline__ void load_group(const QxDev &d, const QxImage &im, const uint32_t *pool, int g,
                                                  int m, int lane) {
    float4 v[4];
    float *row;
    if (g < 3072) {
        // byte tables (core.py:1194-1212): head h, value head x, row rr = pp + 64 * half;
        // columns 2 + 32 half + 4 k + b hold byte b of word h*per + x*per/2 + pp*16 + half*8 + k.
        // The lane's columns 4 lane .. 4 lane + 3 are bytes j = 4q - 2 .. 4q + 1 of the row's eight
        // words (q = lane - 8 half): bytes 2, 3 of word q - 1 and bytes 0, 1 of word q.
        const bool rom = g < 2048;
        const int k0 = 4 * (rom ? g : g - 2048);
        const int h = k0 / 256, x = (k0 / 128) % 2, rr = k0 % 128;
        const int t = (rom ? T_ROM : T_DROM) + h;
        if (shared_table(d, t)) {
            if (!im.write_tables) return;  // the image's copy is (being) written by another machine
            m = (int)im.img;
        }
        row = row_ptr(d, t, x, rr, m);
        const int half = rr >> 6, q = lane - 8 * half;
        const uint32_t len = rom ? im.rom_len : im.drom_words, off = rom ? im.rom_off : im.drom_off;
        const uint32_t base = (uint32_t)(h * 2048 + x * 1024 + (rr & 63) * 16 + half * 8);
        uint32_t wa[4] = {0, 0, 0, 0}, wb[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const uint32_t b = base + 16 * j;
            if (q >= 1 && q <= 8 && b + q - 1 < len) wa[j] = pool[off + b + q - 1];
            if (q >= 0 && q <= 7 && b + q < len) wb[j] = pool[off + b + q];
        }
#pragma unroll
        for (int j = 0; j < 4; j++)
            v[j] = make_float4((float)(wa[j] >> 16 & 0xFF), (float)(wa[j] >> 24), (float)(wb[j] & 0xFF),
                               (float)(wb[j] >> 8 & 0xFF));
    } else if (g < 3584) {
        // digit file: rows rr .. rr + 3 share one word of digits (a byte per row)
        const int k0 = 4 * (g - 3072);
        const int port = k0 / 1024, h = (k0 / 256) % 4, x = (k0 / 128) % 2, rr = k0 % 128;
        row = row_ptr(d, (port ? T_BN2 : T_BN1) + h, x, rr, m);
        const uint32_t dw = im.bn_off != 0xFFFFFFFFu ? pool[im.bn_off + (2 * h + x) * 32 + rr / 4] : 0u;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            // columns 2 .. 5 hold the digit's four bits (lanes 0 and 1)
            const uint32_t bits = lane < 2 ? ((dw >> (8 * j) & 0xF) << 2 >> (4 * lane)) & 15u : 0u;
            v[j] = make_float4((bits & 1) ? A_BIT : 0.f, (bits & 2) ? A_BIT : 0.f, (bits & 4) ? A_BIT : 0.f,
                               (bits & 8) ? A_BIT : 0.f);
        }
    } else {
        // RAM: group u0 = 4 (g - 3584) holds rows r0 .. r0 + 3 of value head x of table tsel;
        // row r of it is word (tsel & 15) | x << 4 | r << 5 | (tsel >> 4) << 12
        const int u0 = 4 * (g - 3584);
        const uint32_t tsel = (uint32_t)u0 >> 8, x = (uint32_t)u0 >> 7 & 1, r0 = (uint32_t)u0 & 127;
        row = row_ptr(d, T_RAM + tsel, x, r0, m);
        const uint32_t wi0 = (tsel & 15) | x << 4 | r0 << 5 | (tsel >> 4) << 12;
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; j++) w[j] = pool[im.ram_off + wi0 + 32 * j];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            // columns 2 .. 33 hold bits 0 .. 31: the lane's columns are bits 4 lane - 2 .. 4 lane + 1;
            // a zero word's row is all zeros (no ballast)
            const uint32_t bits = lane < 9 ? (uint32_t)(((uint64_t)w[j] << 2) >> (4 * lane)) & 15u : 0u;
            v[j] = make_float4((bits & 1) ? A_BIT : 0.f, (bits & 2) ? A_BIT : 0.f, (bits & 4) ? A_BIT : 0.f,
                               (bits & 8) ? A_BIT : 0.f);
            if (lane == 0 && w[j]) { v[j].x = A_REF; v[j].y = A_REF; }
        }
#pragma unroll
        for (int j = 0; j < 4; j++) *reinterpret_cast<float4 *>(row + j * QX_HD + lane * 4) = v[j];
        return;
    }
    if (lane == 0) {
#pragma unroll
        for (int j = 0; j < 4; j++) { v[j].x = A_REF; v[j].y = A_REF; }
    }
#pragma unroll
    for (int j = 0; j < 4; j++) *reinterpret_cast<float4 *>(row + j * QX_HD + lane * 4) = v[j];
}

// One warp per work item; blockIdx.y = machine (row0 + y).  Work items: the row groups, the small
// rows, then the rows no content task writes, four list entries an item (zeros).  Every row of
// the machine's state is written once, so the state needs no clearing beforehand.
__global__ void qx_load_kernel(const __grid_constant__ QxDev d, const QxImage *img, const uint32_t *pool,
                               int32_t row0, int32_t n) {
    const int i = blockIdx.y;
    if (i >= n) return;
    const int m = row0 + i;
    const QxImage &im = img[i];  // read in place (a copy would live in local memory)
    const int lane = threadIdx.x & 31;
    const int warps = blockDim.x / 32, gw = blockIdx.x * warps + (threadIdx.x >> 5);
    const int stride = gridDim.x * warps;
    const int z0 = QX_LOAD_GROUPS + QX_LOAD_SMALL, total = z0 + (d.n_zero_rows + 3) / 4;
    if (d.shared_hl && blockIdx.x == 0 && threadIdx.x == 0) d.img[m] = (int32_t)im.img;
    for (int w = gw; w < total; w += stride) {
        if (w < QX_LOAD_GROUPS) {
            load_group(d, im, pool, w, m, lane);
        } else if (w < z0) {
            float4 v;
            float *row = small_row(d, im, w - QX_LOAD_GROUPS, m, lane, v);
            *reinterpret_cast<float4 *>(row + lane * 4) = v;
        } else {
            const int e0 = 4 * (w - z0);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                if (e0 + j >= d.n_zero_rows) break;
                const uint2 z = d.zero_rows[e0 + j];
                const bool shared = d.shared_hl >> z.x & 1u;
                if (shared && !im.write_tables) continue;
                const size_t c = shared ? (size_t)im.img : (size_t)m;
                float *row = d.S[z.x] + (c * d.V[z.x] * QX_HD + z.y) * QX_HD;
                *reinterpret_cast<float4 *>(row + lane * 4) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    }
}

// Registers (a bit is set when any of its source columns is), PC anchor and n, RAM words of
// machines [row0, row0 + n) into out[n].
__global__ void qx_readback_kernel(const __grid_constant__ QxDev d, int32_t row0, int32_t n, qx_state *out) {
    const int i = blockIdx.x;
    if (i >= n) return;
    const int m = row0 + i;
    qx_state *st = out + i;
    for (int reg = threadIdx.x; reg < 32; reg += blockDim.x) {
        uint32_t v = 0;
        if (reg > 0) {
            const float *row = row_ptr(d, T_REGS, 0, reg, m);
            for (int b = 0; b < 32; b++)
                for (int c = 0; c < 8; c++) {
                    int col = d.reg_cols[b * 8 + c];
                    if (col < 0) break;
                    if (row[col] != 0.0f) { v |= 1u << b; break; }
                }
        }
        st->x[reg] = v;
    }
    if (threadIdx.x == 32) {
        const float *pc = row_ptr(d, T_PC, 0, 0, m);
        uint32_t a = 0;
        for (int b = 0; b < 16; b++)
            if (pc[2 + b] != 0.0f) a |= 1u << b;
        st->anchor = a;
        const float c2 = row_ptr(d, T_COUNT, 0, 0, m)[2];
        st->n = c2 > 0.0f ? (uint32_t)lrintf(log2f(A_BIT / c2)) : 0xFFFFFFFFu;
    }
    for (uint32_t wi = threadIdx.x; wi < RAM_WORDS; wi += blockDim.x) {
        const float *row = row_ptr(d, T_RAM + ((wi & 15) | (wi >> 12) << 4), wi >> 4 & 1, wi >> 5 & 127, m);
        uint32_t v = 0;
        for (int b = 0; b < 32; b++)
            if (__fadd_rn(row[2 + b], row[34 + b]) != 0.0f) v |= 1u << b;
        st->ram[wi] = v;
    }
}

// FNV-1a 64 of (x1..x31, anchor, n, RAM), one thread per machine.
__global__ void qx_checksum_kernel(const qx_state *st, int32_t n, uint64_t *out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const qx_state *s = st + i;
    uint64_t h = 0xcbf29ce484222325ULL;
    auto mix = [&](uint32_t w) {
        for (int b = 0; b < 4; b++) {
            h ^= (w >> (8 * b)) & 0xFFu;
            h *= 0x100000001b3ULL;
        }
    };
    for (int r = 1; r < 32; r++) mix(s->x[r]);
    mix(s->anchor);
    mix(s->n);
    for (int w = 0; w < (int)RAM_WORDS; w++) mix(s->ram[w]);
    out[i] = h;
}

// Zero the lag histories of machines [row0, row0 + n).
__global__ void qx_reset_kernel(float *H, uint32_t ne, uint32_t bpad, int32_t row0, int32_t n) {
    const size_t total = (size_t)3 * ne * n;
    for (size_t k = blockIdx.x * (size_t)blockDim.x + threadIdx.x; k < total; k += (size_t)gridDim.x * blockDim.x) {
        const size_t e = k / n, r = k % n;
        H[e * bpad + row0 + r] = 0.0f;
    }
}
