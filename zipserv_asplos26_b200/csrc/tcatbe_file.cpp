// On-disk container for one TCA-TBE compressed matrix (file format version 1).
//
// The reference has no serialised form: its benchmarks compress weights at
// start-up from the dense BF16 checkpoint (kernel_benchmark/
// bench_zipserv_gemm_sweep.cu:290-345, scripts/export_llama31_70b_weights.py
// exports only dense tensors). This container stores the arrays the GPU path
// reads -- the same bytes the encoders produce (csrc/L_API.cu:559-771 layout) --
// so a server can load compressed weights without re-encoding them.
//
// Layout (little-endian, all offsets in bytes from the start of the file):
//   0    char[8]  magic "ZSTCATBE"
//   8    u32      version (1)
//   12   u32      header bytes (512; arrays start at or after it)
//   16   i64      rows, i64 cols
//   32   i32      start_exp, max_hf, max_full, has_st_counts
//   48   i32[7]   top exponents, i32 reserved
//   80   i64      total_hf, i64 total_full
//   96   u32      array count (8), u32 reserved
//   104  8 x {u32 id, u32 element bytes, u64 element count, u64 offset,
//              u32 crc32, u32 reserved} (32 bytes each)
//   then the arrays, each starting on a 256-byte boundary, in id order:
//     0 sign/mantissa stream  u8   total_hf
//     1 fallback stream       u16  total_full
//     2-4 bitmaps 1-3         u64  #ST = rows*cols/64 each
//     5 small-tile counts     i32  2*#ST (0 when absent; no kernel reads them)
//     6 median-tile offsets   i32  2*#MT, #MT = #ST/16
//     7 global-tile offsets   i32  2*(#GT+1), #GT = rows*cols/4096
// The CRC-32 (IEEE 802.3 polynomial, reflected, as in zlib and PNG) of every
// array is checked on load.
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#include "zipserv_b200.h"

namespace {

constexpr char kMagic[8] = {'Z', 'S', 'T', 'C', 'A', 'T', 'B', 'E'};
constexpr uint32_t kVersion = 1;
constexpr uint32_t kHeaderBytes = 512;
constexpr int kArrays = 8;
constexpr int kErrInvalid = 1;      // cudaErrorInvalidValue
constexpr int kErrNoFile = 301;     // cudaErrorFileNotFound
constexpr int kErrIo = 999;         // cudaErrorUnknown

struct Entry {
    uint32_t id, elem_bytes;
    uint64_t count, offset;
    uint32_t crc, reserved;
};
static_assert(sizeof(Entry) == 32, "array table entry is 32 bytes");

struct Header {
    char magic[8];
    uint32_t version, header_bytes;
    int64_t rows, cols;
    int32_t start_exp, max_hf, max_full, has_st;
    int32_t top[7], reserved0;
    int64_t total_hf, total_full;
    uint32_t n_arrays, reserved1;
    Entry e[kArrays];
};
static_assert(sizeof(Header) == 104 + kArrays * 32, "header layout");
static_assert(sizeof(Header) <= kHeaderBytes, "header fits its reserved bytes");

// Table-driven CRC-32 (reflected polynomial 0xEDB88320); the table is built
// from the polynomial once (thread-safe static initialisation).
struct CrcTable {
    uint32_t t[256];
    CrcTable() {
        for (uint32_t i = 0; i < 256; ++i) {
            uint32_t c = i;
            for (int k = 0; k < 8; ++k) c = (c & 1u) ? (0xEDB88320u ^ (c >> 1)) : (c >> 1);
            t[i] = c;
        }
    }
};

uint32_t crc32(const void* data, size_t n) {
    static const CrcTable tab;
    const uint32_t* table = tab.t;
    uint32_t c = 0xFFFFFFFFu;
    const uint8_t* p = static_cast<const uint8_t*>(data);
    for (size_t i = 0; i < n; ++i) c = table[(c ^ p[i]) & 0xFFu] ^ (c >> 8);
    return c ^ 0xFFFFFFFFu;
}

// Element sizes and counts of the eight arrays for a given info.
bool array_shapes(const ZsTcatbeInfo& in, uint32_t esz[kArrays], uint64_t cnt[kArrays]) {
    if (in.rows <= 0 || in.cols <= 0 || in.rows % 64 || in.cols % 64) return false;
    if (in.total_hf < 0 || in.total_full < 0 || in.total_hf > in.rows * in.cols ||
        in.total_full > in.rows * in.cols)
        return false;
    if (in.max_hf < 0 || in.max_full < 0 || in.max_hf > 4096 + 15 || in.max_full > 4096 + 7) return false;
    const uint64_t nst = (uint64_t)in.rows * (uint64_t)in.cols / 64, nmt = nst / 16, ngt = nst / 64;
    const uint32_t e[kArrays] = {1, 2, 8, 8, 8, 4, 4, 4};
    const uint64_t c[kArrays] = {(uint64_t)in.total_hf, (uint64_t)in.total_full, nst, nst, nst,
                                 in.has_st_counts ? 2 * nst : 0, 2 * nmt, 2 * (ngt + 1)};
    for (int i = 0; i < kArrays; ++i) { esz[i] = e[i]; cnt[i] = c[i]; }
    return true;
}

struct File {
    FILE* f = nullptr;
    ~File() { if (f) fclose(f); }
};

int read_header(FILE* f, Header* h) {
    if (fread(h, sizeof(Header), 1, f) != 1) return kErrIo;
    if (memcmp(h->magic, kMagic, 8) != 0 || h->version != kVersion || h->header_bytes < sizeof(Header) ||
        h->n_arrays != kArrays)
        return kErrInvalid;
    return 0;
}

void info_from_header(const Header& h, ZsTcatbeInfo* in) {
    in->rows = h.rows;
    in->cols = h.cols;
    in->start_exp = h.start_exp;
    in->max_hf = h.max_hf;
    in->max_full = h.max_full;
    for (int i = 0; i < 7; ++i) in->top[i] = h.top[i];
    in->total_hf = h.total_hf;
    in->total_full = h.total_full;
    in->has_st_counts = h.has_st;
}

}  // namespace

extern "C" int zs_tcatbe_save(const char* path, const ZsTcatbeInfo* info, const uint8_t* sm, const uint16_t* full,
                              const uint64_t* b1, const uint64_t* b2, const uint64_t* b3, const int* st_counts,
                              const int* mt_off, const int* gt_off) {
    if (!path || !info) return kErrInvalid;
    uint32_t esz[kArrays];
    uint64_t cnt[kArrays];
    if (!array_shapes(*info, esz, cnt)) return kErrInvalid;
    const void* src[kArrays] = {sm, full, b1, b2, b3, st_counts, mt_off, gt_off};
    for (int i = 0; i < kArrays; ++i)
        if (cnt[i] && !src[i]) return kErrInvalid;
    Header h;
    memset(&h, 0, sizeof(h));
    memcpy(h.magic, kMagic, 8);
    h.version = kVersion;
    h.header_bytes = kHeaderBytes;
    h.rows = info->rows;
    h.cols = info->cols;
    h.start_exp = info->start_exp;
    h.max_hf = info->max_hf;
    h.max_full = info->max_full;
    h.has_st = info->has_st_counts ? 1 : 0;
    for (int i = 0; i < 7; ++i) h.top[i] = info->top[i];
    h.total_hf = info->total_hf;
    h.total_full = info->total_full;
    h.n_arrays = kArrays;
    uint64_t off = kHeaderBytes;
    for (int i = 0; i < kArrays; ++i) {
        off = (off + 255) / 256 * 256;
        h.e[i].id = (uint32_t)i;
        h.e[i].elem_bytes = esz[i];
        h.e[i].count = cnt[i];
        h.e[i].offset = off;
        h.e[i].crc = cnt[i] ? crc32(src[i], cnt[i] * esz[i]) : 0u;
        off += cnt[i] * esz[i];
    }
    File fh;
    fh.f = fopen(path, "wb");
    if (!fh.f) return kErrNoFile;
    std::vector<uint8_t> pad(kHeaderBytes, 0);
    memcpy(pad.data(), &h, sizeof(h));
    if (fwrite(pad.data(), 1, kHeaderBytes, fh.f) != kHeaderBytes) return kErrIo;
    uint64_t pos = kHeaderBytes;
    static const uint8_t zeros[256] = {};
    for (int i = 0; i < kArrays; ++i) {
        if (h.e[i].offset > pos) {
            const size_t gap = (size_t)(h.e[i].offset - pos);
            if (fwrite(zeros, 1, gap, fh.f) != gap) return kErrIo;
            pos += gap;
        }
        const size_t bytes = (size_t)(cnt[i] * esz[i]);
        if (bytes && fwrite(src[i], 1, bytes, fh.f) != bytes) return kErrIo;
        pos += bytes;
    }
    if (fflush(fh.f) != 0) return kErrIo;
    return 0;
}

extern "C" int zs_tcatbe_read_info(const char* path, ZsTcatbeInfo* info) {
    if (!path || !info) return kErrInvalid;
    File fh;
    fh.f = fopen(path, "rb");
    if (!fh.f) return kErrNoFile;
    Header h;
    if (int r = read_header(fh.f, &h)) return r;
    info_from_header(h, info);
    uint32_t esz[kArrays];
    uint64_t cnt[kArrays];
    if (!array_shapes(*info, esz, cnt)) return kErrInvalid;
    for (int i = 0; i < kArrays; ++i)
        if (h.e[i].id != (uint32_t)i || h.e[i].elem_bytes != esz[i] || h.e[i].count != cnt[i]) return kErrInvalid;
    return 0;
}

extern "C" int zs_tcatbe_load(const char* path, ZsTcatbeInfo* info, uint8_t* sm, uint16_t* full, uint64_t* b1,
                              uint64_t* b2, uint64_t* b3, int* st_counts, int* mt_off, int* gt_off) {
    if (!path || !info) return kErrInvalid;
    File fh;
    fh.f = fopen(path, "rb");
    if (!fh.f) return kErrNoFile;
    Header h;
    if (int r = read_header(fh.f, &h)) return r;
    ZsTcatbeInfo in;
    info_from_header(h, &in);
    uint32_t esz[kArrays];
    uint64_t cnt[kArrays];
    if (!array_shapes(in, esz, cnt)) return kErrInvalid;
    void* dst[kArrays] = {sm, full, b1, b2, b3, st_counts, mt_off, gt_off};
    for (int i = 0; i < kArrays; ++i) {
        if (h.e[i].id != (uint32_t)i || h.e[i].elem_bytes != esz[i] || h.e[i].count != cnt[i]) return kErrInvalid;
        if (cnt[i] && !dst[i] && i != 5) return kErrInvalid;   // small-tile counts may be skipped
    }
    for (int i = 0; i < kArrays; ++i) {
        if (!cnt[i] || !dst[i]) continue;
        const size_t bytes = (size_t)(cnt[i] * esz[i]);
        if (fseek(fh.f, (long)h.e[i].offset, SEEK_SET) != 0) return kErrIo;
        if (fread(dst[i], 1, bytes, fh.f) != bytes) return kErrIo;
        if (crc32(dst[i], bytes) != h.e[i].crc) return kErrInvalid;
    }
    // The offsets must describe streams the decoders can stage: the global
    // offsets start at zero, never decrease, give each tile at most max_hf hf
    // bytes and max_full fallback elements (padded to 16 bytes / 8 elements)
    // and end at the stream totals; each tile's median-tile offsets start at
    // zero, never decrease and stay inside the tile. (A file whose CRCs match
    // but whose offsets do not would otherwise send the GPU decoders past the
    // staged streams.)
    const uint64_t ngt = (uint64_t)in.rows * (uint64_t)in.cols / 4096;
    const int64_t hcap = ((int64_t)in.max_hf + 15) / 16 * 16, fcap = ((int64_t)in.max_full + 7) / 8 * 8;
    if (gt_off[0] != 0 || gt_off[1] != 0) return kErrInvalid;
    for (uint64_t g = 0; g < ngt; ++g) {
        const int64_t dh = (int64_t)gt_off[2 * g + 2] - gt_off[2 * g], df = (int64_t)gt_off[2 * g + 3] - gt_off[2 * g + 1];
        if (dh < 0 || df < 0 || dh > hcap || df > fcap) return kErrInvalid;
        if (mt_off) {
            const int* m = mt_off + 8 * g;
            if (m[0] != 0 || m[1] != 0) return kErrInvalid;
            for (int w = 1; w < 4; ++w)
                if (m[2 * w] < m[2 * w - 2] || m[2 * w + 1] < m[2 * w - 1] || m[2 * w] > dh || m[2 * w + 1] > df)
                    return kErrInvalid;
        }
    }
    if ((int64_t)gt_off[2 * ngt] != in.total_hf || (int64_t)gt_off[2 * ngt + 1] != in.total_full) return kErrInvalid;
    *info = in;
    return 0;
}
