// Host-built arithmetic tables of the LNS hot path.
//
// Every table the kernels read is computed here, on the host, once per
// process, and uploaded per device by lnsb_upload_tables.  The device never
// evaluates a transcendental function of its own for xlns16, so a kernel's
// result depends only on integer arithmetic and these tables.
//
// Definitions (the reference's configuration: xlns16_table + xlns16_alt,
// xlns32_alt; lns-backend/src/lns-ops.cpp:43-53, lns-backend/src/CMakeLists.txt:13):
//   sb(n) = log2(1 + 2^(-n/128)), db(n) = log2(1 - 2^(-n/128)) at F=7, n = 0..1280
//   (essential zero 0x500), rounded with (int)(v + 0.5) -- db through
//   log2(2^(n/128) - 1), which is negative below n = 128.
//   float -> xlns16: 65536-entry table over the float's upper 16 bits.
//   xlns16 -> float: 2^(l/128) to 7 significant digits.
//   xlns32: table sb with linear interpolation, cotransformed db (F=23).
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

namespace lnsb {

// Layout of the xlns16 Gaussian-log table as kernels keep it in shared
// memory: 16-bit entries, logs scaled by 2 so a byte offset is the index.
//   bytes [0,    2564): sb adjustment * 2 at byte 2n, n = 0..1281 (n = 1281 -> 0)
//   bytes [4096, 6660): db adjustment * 2 at byte 4096 + 2n (n = 0 -> -65536 sentinel
//                       is not representable in 16 bits; n = 0 is handled by the caller)
constexpr int k16_sign_off   = 4096;   // byte offset of the db half == sign flag value
constexpr int k16_tab_bytes  = 6660;
constexpr int k16_tab_bytes16 = (k16_tab_bytes + 15) / 16 * 16;   // the device copy, padded for 16-byte copies
constexpr int k16_ess        = 1280;
constexpr int k16_ess_clamp2 = 2 * (k16_ess + 1);   // 2562: clamp of 2n, entry is 0

// Monte fine tables: sb/db at 8 extra fraction bits, n = 0..2303
constexpr int k16_monte_n = 2304;

// "Key" form of the xlns16 Gaussian-log table, for the base-mode mul_mat fast
// path.  A value is carried as key = 16 * log + 4 * (value < 0 ? 1 : 0); for
// two keys a (accumulator) and p (term), |a - p| is 16n (same signs) or
// 16n +- 4 (opposite signs), n = |log a - log p|.  The table is indexed by
// that difference as a byte offset: 32-bit entry at byte 16n holds 16 * sb(n),
// at bytes 16n - 4 and 16n + 4 16 * db(n) (n >= 1), at byte 4 the exact-
// cancellation sentinel, and 0 from n = 1281 on (essential zero).
constexpr int k16_key_max   = 16 * (k16_ess + 1) + 4;          // largest index used
constexpr int k16_key_bytes = (k16_key_max + 4 + 15) / 16 * 16;  // 20512
constexpr int k16_key_cancel = -(1 << 30);

// Signed image of key16 for the latency kernels: the 32-bit entry for a key
// difference D (a multiple of 4, |D| <= k16_key_max) sits at byte
// k16_key_max + D, so a clamped signed difference indexes it directly.
constexpr int k16s_bytes = (2 * k16_key_max + 4 + 15) / 16 * 16;   // 41008

// The same key indexing over the Monte fine tables, for the Monte mul_mat fast
// path: 32-bit entry at byte 16n holds the fine sb(n) (x 256), at bytes 16n -
// 4 and 16n + 4 the fine db(n) (n >= 1), at byte 4 the cancellation sentinel,
// and 0 from n = k16_monte_n on (the fine tables' end).
constexpr int k16m_key_max   = 16 * k16_monte_n + 4;
constexpr int k16m_key_bytes = (k16m_key_max + 4 + 15) / 16 * 16;   // 36880

// xlns32 interpolation geometry (units: 2^-23 octave): sb knots every 2^-9
// octave on [0, 26], db knots every 2^-9 octave on [1, 26], knots truncated
// toward zero, interpolation floored.
constexpr uint32_t k32_one = 1u << 23;
constexpr uint32_t k32_ess = 26u << 23;
constexpr int      k32_sh  = 14;                    // knot spacing 2^14 units
constexpr int      k32_sb_knots = (26 << 9) + 1;   // z = n << 14, n = 0..13312
constexpr int      k32_db_knots = (25 << 9) + 1;   // z = (1 << 23) + (n << 14), n = 0..12800

// Flat xlns32 addition image (int32 words): everything one xlns32 addition
// reads, in one block that a kernel keeps in shared memory.
//   [k32f_sb, +13314)  sb knots, then a 0 (the right knot of z = ess)
//   [k32f_db, +12802)  db knots, then a 0; the knot of z sits at word
//                      k32f_db0 + (z >> 14) for z >= 1 octave
//   [k32f_lo, +4096)   db(d) for d = 0..4095 (cotransformation, low part)
//   [k32f_hi, +2048)   db(j << 12) for j = 0..2047 (cotransformation, high part)
//                      index 0 of both holds k32f_none, which makes the
//                      cotransformation's special cases (d < 4096 or d a
//                      multiple of 4096) fall out of the general formula
// Every interpolation product (right - left) * f fits in 32 bits (checked
// when the image is built).
constexpr int     k32f_sb      = 0;
constexpr int     k32f_db      = 13316;
constexpr int     k32f_db0     = k32f_db - 512;
constexpr int     k32f_lo      = 26120;
constexpr int     k32f_hi      = 30216;
constexpr int     k32f_words   = 32264;          // multiple of 4 (16-byte copies)
constexpr int     k32f_sb_bytes16 = k32f_db * 4;  // the sb knots, in 16-byte pieces
constexpr int32_t k32f_none    = -(1 << 30);

struct host_tables {
    // xlns16
    std::vector<int16_t>  sbdb16;      // k16_tab_bytes / 2 entries, smem image
    std::vector<uint16_t> conv16;      // 131072, indexed by a float's bits >> 15
    std::vector<float>    dec16;       // 65536
    std::vector<uint16_t> exp16;       // 65536
    std::vector<uint16_t> sig16;       // 65536
    std::vector<int16_t>  monte16;     // [2 * k16_monte_n]: sb fine, then db fine
    std::vector<int32_t>  key16;       // k16_key_bytes / 4 entries, see k16_key_max
    std::vector<int32_t>  mkey16;      // k16m_key_bytes / 4 entries, see k16m_key_max
    std::vector<int32_t>  key16s;      // k16s_bytes / 4 entries, see k16s_bytes
    // xlns32
    std::vector<int32_t>  sb32;        // k32_sb_knots + 1 (a trailing 0)
    std::vector<int32_t>  db32;        // k32_db_knots + 1 (a trailing 0)
    std::vector<int32_t>  db32_hi;     // 2048
    std::vector<int32_t>  db32_lo;     // 4096
    std::vector<int32_t>  flat32;      // k32f_words, see k32f_sb
    std::vector<uint32_t> logm32;      // 2^23 (LNS32 conversion), may be empty
    std::vector<float>    expm32;      // 2^23 (LNS32 decode), may be empty
    std::vector<int32_t>  lpvip_db;    // 2^23 (LPVIP singular branch), may be empty
    std::vector<uint16_t> lfsr_log;    // 65536 (Monte jump-ahead)
    std::vector<uint16_t> lfsr_alog;   // 65535
};

// e^x in double and float, the host twins of the device's lnsb_exp_d and
// lnsb_expf (bit-identical: the same correctly rounded operations)
double host_exp_d(double x);
float host_expf(float x);

// Builds (once) and returns the tables.  need32: LNS32 conversion tables;
// need_lpvip: the 2^23-entry LPVIP singular-branch table.
const host_tables & get_host_tables(bool need32, bool need_lpvip);

}  // namespace lnsb
