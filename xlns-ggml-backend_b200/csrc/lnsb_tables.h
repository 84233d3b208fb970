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

// xlns32 interpolation geometry (units: 2^-23 octave)
struct seg32 { uint32_t lo, hi; int shift; int base; };
constexpr uint32_t k32_one = 1u << 23;
constexpr uint32_t k32_ess = 26u << 23;

struct host_tables {
    // xlns16
    std::vector<int16_t>  sbdb16;      // k16_tab_bytes / 2 entries, smem image
    std::vector<uint16_t> conv16;      // 65536
    std::vector<float>    dec16;       // 65536
    std::vector<uint16_t> exp16;       // 65536
    std::vector<int16_t>  monte16;     // [2 * k16_monte_n]: sb fine, then db fine
    std::vector<int32_t>  key16;       // k16_key_bytes / 4 entries, see k16_key_max
    // xlns32
    seg32 sb_seg[2], db_seg[4];
    std::vector<int32_t>  sb32, db32;  // concatenated knots
    std::vector<int32_t>  db32_hi;     // 2048
    std::vector<int32_t>  db32_lo;     // 4096
    std::vector<uint32_t> logm32;      // 2^23 (LNS32 conversion), may be empty
    std::vector<float>    expm32;      // 2^23 (LNS32 decode), may be empty
    std::vector<int32_t>  lpvip_db;    // 2^23 (LPVIP singular branch), may be empty
    std::vector<uint16_t> lfsr_log;    // 65536 (Monte jump-ahead)
    std::vector<uint16_t> lfsr_alog;   // 65535
};

// Builds (once) and returns the tables.  need32: LNS32 conversion tables;
// need_lpvip: the 2^23-entry LPVIP singular-branch table.
const host_tables & get_host_tables(bool need32, bool need_lpvip);

}  // namespace lnsb
