// tk_tq.cu -- the `.tq` quantized-base file: reader and writer (host code).
//
// Format (the reference's tq_load, tier/tier.cpp:274-292, and its writers
// quant_main, tier/tier.cpp:2698-2746, and write_tq, tier/quant.py:60-105):
//   bytes [0, hb): text header, NUL-padded:
//     "TQB1 <hb> <n>\n", optional "#key value\n" lines, then one line per
//     matrix "<name> <type> <rows> <cols> <offset> <bytes> <err>\n"
//     (err: relative RMS quantization error, or -1 when unknown);
//     hb = (n * 200 + 4096 + 4095) / 4096 * 4096.
//   each matrix: rows * row_bytes(type, cols) bytes of the reference's block
//   rows at its offset; offsets start at hb and are 4096-aligned.
// The reader applies the reference's checks: magic and 64 <= hb <= 64 MiB;
// lines that do not parse into six fields are skipped, a known-looking line
// with an unknown type, a column count off the block size or a byte count
// that is not rows * row_bytes rejects the file.
#include "tk_internal.h"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <sstream>
#include <string>
#include <vector>

struct tk_tq {
    std::string path;
    struct Ent {
        std::string name;
        int qtype, rows, cols;
        uint64_t offset, bytes;
        double err;
    };
    std::vector<Ent> ents;
};

namespace tk {

// The reference's type table (tier/quant.h:25-31): code, name, elements per
// block, bytes per block.  It is the file format's vocabulary, so it is
// kept entry for entry.
struct QName {
    int code;
    const char* name;
    int blk, bytes;
};
static const QName kNames[] = {
    {0, "F32", 1, 4},       {1, "F16", 1, 2},        {30, "BF16", 1, 2},      {2, "Q4_0", 32, 18},
    {3, "Q4_1", 32, 20},    {6, "Q5_0", 32, 22},     {7, "Q5_1", 32, 24},     {8, "Q8_0", 32, 34},
    {10, "Q2_K", 256, 84},  {11, "Q3_K", 256, 110},  {12, "Q4_K", 256, 144},  {13, "Q5_K", 256, 176},
    {14, "Q6_K", 256, 210}, {16, "IQ2_XXS", 256, 66}, {17, "IQ2_XS", 256, 74}, {22, "IQ2_S", 256, 82},
    {18, "IQ3_XXS", 256, 98}, {21, "IQ3_S", 256, 110}, {19, "IQ1_S", 256, 50}, {29, "IQ1_M", 256, 56},
    {20, "IQ4_NL", 32, 18}, {23, "IQ4_XS", 256, 136}, {34, "TQ1_0", 256, 54},  {35, "TQ2_0", 256, 66},
    {39, "MXFP4", 32, 17},  {200, "NF4", 64, 36},    {201, "FP4", 64, 36},
};
static const QName* qname(int code) {
    for (const QName& q : kNames)
        if (q.code == code) return &q;
    return nullptr;
}
static const QName* qname(const char* s) {
    for (const QName& q : kNames)
        if (!strcmp(q.name, s)) return &q;
    return nullptr;
}

static bool pread_all(int fd, void* dst, size_t n, uint64_t off) {
    uint8_t* p = static_cast<uint8_t*>(dst);
    while (n) {
        const ssize_t r = pread(fd, p, n, (off_t)off);
        if (r <= 0) return false;
        p += r;
        n -= (size_t)r;
        off += (uint64_t)r;
    }
    return true;
}
static bool pwrite_all(int fd, const void* src, size_t n, uint64_t off) {
    const uint8_t* p = static_cast<const uint8_t*>(src);
    while (n) {
        const ssize_t r = pwrite(fd, p, n, (off_t)off);
        if (r <= 0) return false;
        p += r;
        n -= (size_t)r;
        off += (uint64_t)r;
    }
    return true;
}

}  // namespace tk

using namespace tk;

extern "C" {

int tk_qtype_from_name(const char* name) {
    const QName* q = name ? qname(name) : nullptr;
    return q ? q->code : -1;
}

const char* tk_qtype_name(int qtype) {
    const QName* q = qname(qtype);
    return q ? q->name : nullptr;
}

tk_status tk_tq_open(const char* path, tk_tq** out) {
    if (!path || !out) return fail(TK_ERR_INVALID, "tk_tq_open: null argument");
    *out = nullptr;
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return fail(TK_ERR_INVALID, std::string("tk_tq_open: cannot open ") + path);
    char first[128] = {0};
    const ssize_t got = pread(fd, first, sizeof first - 1, 0);
    size_t hb = 0, n = 0;
    if (got < 8 || sscanf(first, "TQB1 %zu %zu", &hb, &n) != 2 || hb < 64 || hb > (64ull << 20)) {
        close(fd);
        return fail(TK_ERR_INVALID, std::string("tk_tq_open: ") + path + " is not a TQB1 quantized base");
    }
    std::string h(hb, '\0');
    const bool ok = pread_all(fd, &h[0], hb, 0);
    close(fd);
    if (!ok) return fail(TK_ERR_INVALID, std::string("tk_tq_open: ") + path + ": header truncated");
    std::istringstream is(h.substr(0, h.find('\0')));
    std::string line;
    std::getline(is, line);   // the TQB1 line
    tk_tq* t = new tk_tq();
    t->path = path;
    while (std::getline(is, line)) {
        if (line.empty() || line[0] == '#') continue;
        char nm[256], ty[32];
        int rows, cols;
        unsigned long long off, sz;
        double err = -1.0;
        const int k = sscanf(line.c_str(), "%255s %31s %d %d %llu %llu %lf", nm, ty, &rows, &cols, &off, &sz, &err);
        if (k < 6) continue;
        const QName* q = qname(ty);
        if (!q || rows < 0 || cols <= 0 || cols % q->blk || (uint64_t)(cols / q->blk) * q->bytes * (uint64_t)rows != sz) {
            delete t;
            return fail(TK_ERR_INVALID, std::string("tk_tq_open: matrix ") + nm + " of type " + ty + " does not parse");
        }
        t->ents.push_back({nm, q->code, rows, cols, off, sz, k >= 7 ? err : -1.0});
    }
    *out = t;
    return TK_OK;
}

void tk_tq_close(tk_tq* tq) { delete tq; }

int tk_tq_count(const tk_tq* tq) { return tq ? (int)tq->ents.size() : 0; }

int tk_tq_find(const tk_tq* tq, const char* name) {
    if (!tq || !name) return -1;
    for (size_t i = 0; i < tq->ents.size(); ++i)
        if (tq->ents[i].name == name) return (int)i;
    return -1;
}

tk_status tk_tq_entry(const tk_tq* tq, int i, const char** name, int* qtype, int* rows, int* cols, uint64_t* offset,
                      uint64_t* bytes, double* err) {
    if (!tq || i < 0 || i >= (int)tq->ents.size()) return fail(TK_ERR_INVALID, "tk_tq_entry: index out of range");
    const tk_tq::Ent& e = tq->ents[i];
    if (name) *name = e.name.c_str();
    if (qtype) *qtype = e.qtype;
    if (rows) *rows = e.rows;
    if (cols) *cols = e.cols;
    if (offset) *offset = e.offset;
    if (bytes) *bytes = e.bytes;
    if (err) *err = e.err;
    return TK_OK;
}

tk_status tk_tq_read(const tk_tq* tq, int i, void* dst, int dst_on_device, void* stream) {
    if (!tq || !dst || i < 0 || i >= (int)tq->ents.size()) return fail(TK_ERR_INVALID, "tk_tq_read: bad argument");
    const tk_tq::Ent& e = tq->ents[i];
    const int fd = open(tq->path.c_str(), O_RDONLY);
    if (fd < 0) return fail(TK_ERR_INVALID, "tk_tq_read: cannot open " + tq->path);
    if (!dst_on_device) {
        const bool ok = pread_all(fd, dst, e.bytes, e.offset);
        close(fd);
        return ok ? TK_OK : fail(TK_ERR_INVALID, "tk_tq_read: " + e.name + " truncated");
    }
    // to the device through a pinned staging buffer, 32 MiB at a time
    const size_t chunk = 32u << 20;
    void* stage = nullptr;
    cudaError_t ce = cudaHostAlloc(&stage, chunk, cudaHostAllocDefault);
    if (ce != cudaSuccess) {
        close(fd);
        return cuda_fail(ce, "tk_tq_read: pinned buffer");
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    tk_status st = TK_OK;
    for (uint64_t done = 0; done < e.bytes && st == TK_OK; done += chunk) {
        const size_t n = (size_t)(e.bytes - done < chunk ? e.bytes - done : chunk);
        if (!pread_all(fd, stage, n, e.offset + done)) {
            st = fail(TK_ERR_INVALID, "tk_tq_read: " + e.name + " truncated");
            break;
        }
        ce = cudaMemcpyAsync(static_cast<uint8_t*>(dst) + done, stage, n, cudaMemcpyHostToDevice, s);
        if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);   // the stage is reused
        if (ce != cudaSuccess) st = cuda_fail(ce, "tk_tq_read: copy");
    }
    cudaFreeHost(stage);
    close(fd);
    return st;
}

tk_status tk_tq_write(const char* path, int n, const char* const* names, const int* qtypes, const int* rows,
                      const int* cols, const void* const* data, const double* errs, const char* meta) {
    if (!path || n < 0 || (n > 0 && (!names || !qtypes || !rows || !cols || !data)))
        return fail(TK_ERR_INVALID, "tk_tq_write: null argument");
    const size_t hb = ((size_t)n * 200 + 4096 + 4095) / 4096 * 4096;
    std::vector<uint64_t> off(n), size(n);
    uint64_t pos = hb;
    std::string h = "TQB1 " + std::to_string(hb) + " " + std::to_string(n) + "\n";
    if (meta && *meta) {
        h += meta;
        if (h.back() != '\n') h += '\n';
    }
    char b[512];
    for (int i = 0; i < n; ++i) {
        const QName* q = qname(qtypes[i]);
        if (!q || !names[i] || rows[i] < 0 || cols[i] <= 0 || cols[i] % q->blk || strchr(names[i], ' '))
            return fail(TK_ERR_INVALID, std::string("tk_tq_write: matrix ") + (names[i] ? names[i] : "?") +
                                            ": unknown type, bad shape or a space in the name");
        size[i] = (uint64_t)(cols[i] / q->blk) * q->bytes * (uint64_t)rows[i];
        off[i] = pos;
        pos += (size[i] + 4095) / 4096 * 4096;
        if (errs)
            snprintf(b, sizeof b, "%s %s %d %d %llu %llu %.6f\n", names[i], q->name, rows[i], cols[i],
                     (unsigned long long)off[i], (unsigned long long)size[i], errs[i]);
        else
            snprintf(b, sizeof b, "%s %s %d %d %llu %llu -1\n", names[i], q->name, rows[i], cols[i],
                     (unsigned long long)off[i], (unsigned long long)size[i]);
        h += b;
    }
    if (h.size() >= hb) return fail(TK_ERR_INVALID, "tk_tq_write: header does not fit");
    h.resize(hb, '\0');
    const std::string tmp = std::string(path) + ".part";
    const int fd = open(tmp.c_str(), O_RDWR | O_CREAT | O_TRUNC, 0644);
    if (fd < 0) return fail(TK_ERR_INVALID, "tk_tq_write: cannot create " + tmp);
    bool ok = ftruncate(fd, (off_t)pos) == 0 && pwrite_all(fd, h.data(), hb, 0);
    std::vector<uint8_t> host;
    for (int i = 0; i < n && ok; ++i) {
        cudaPointerAttributes a;
        const bool on_dev = cudaPointerGetAttributes(&a, data[i]) == cudaSuccess && a.type == cudaMemoryTypeDevice;
        cudaGetLastError();   // a host pointer may leave an error state behind
        if (!on_dev) {
            ok = pwrite_all(fd, data[i], size[i], off[i]);
            continue;
        }
        const size_t chunk = 32u << 20;
        host.resize(chunk);
        for (uint64_t done = 0; done < size[i] && ok; done += chunk) {
            const size_t m = (size_t)(size[i] - done < chunk ? size[i] - done : chunk);
            ok = cudaMemcpy(host.data(), static_cast<const uint8_t*>(data[i]) + done, m, cudaMemcpyDeviceToHost) ==
                     cudaSuccess &&
                 pwrite_all(fd, host.data(), m, off[i] + done);
        }
    }
    ok = ok && fsync(fd) == 0;
    close(fd);
    if (!ok || rename(tmp.c_str(), path) != 0) {
        unlink(tmp.c_str());
        return fail(TK_ERR_INVALID, std::string("tk_tq_write: writing ") + path + " failed");
    }
    return TK_OK;
}

}  // extern "C"
