// Safetensors reader: the on-disk container of MLX checkpoints, mapped read-only and copied
// to device buffers unchanged (the packed codes, scales and biases on disk are already the
// operator layout).
//
// Replaces the array loading that attaches checkpoint tensors to the prebuilt packed
// modules (loadArrays in Sources/Qwen38Core/FlashNext/Qwen4ExpCheckpointLayerLoader.swift:74
// and Sources/Qwen38Core/Bonsai2/Qwen38Bonsai2Container.swift:30, :87).  The file format
// is the published safetensors layout (huggingface/safetensors; the reader checked against
// here is the Python package 0.7.0): an 8-byte little-endian header length n, n bytes of
// UTF-8 JSON mapping each tensor name to {"dtype", "shape", "data_offsets": [begin, end]}
// (offsets relative to the byte buffer after the header, which they must tile exactly, in
// some order, without gaps or overlaps) plus an optional "__metadata__" string map.
//
// Host code only, apart from the copies.  A device copy moves a 2-D sub-block (rows x
// a byte range of each row, e.g. one tensor-parallel shard) through two pinned staging
// halves: the host gathers one half while the other half's copy is in flight.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <unordered_map>
#include <utility>
#include <vector>

#include "q38_internal.h"

namespace {

struct StTensor {
    std::string name, dtype;
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0;
};

thread_local std::string g_open_error;

int dtype_size(const std::string& d) {
    static const std::pair<const char*, int> table[] = {
        {"BOOL", 1}, {"U8", 1}, {"I8", 1}, {"F8_E5M2", 1}, {"F8_E4M3", 1}, {"I16", 2}, {"U16", 2},
        {"F16", 2},  {"BF16", 2}, {"I32", 4}, {"U32", 4}, {"F32", 4}, {"F64", 8}, {"I64", 8}, {"U64", 8}};
    for (const auto& e : table)
        if (d == e.first) return e.second;
    return 0;
}

// Strict JSON reader for the header: objects, arrays, strings (all escapes, \u with
// surrogate pairs to UTF-8), non-negative integers; other values are skipped where the
// format allows unknown entries.
class Json {
public:
    Json(const char* p, const char* e) : p_(p), e_(e) {}
    std::string error;

    void ws() {
        while (p_ < e_ && (*p_ == ' ' || *p_ == '\t' || *p_ == '\n' || *p_ == '\r')) ++p_;
    }
    bool peek(char c) {
        ws();
        return p_ < e_ && *p_ == c;
    }
    bool take(char c) {
        if (!peek(c)) return fail(std::string("expected '") + c + "'");
        ++p_;
        return true;
    }
    bool at_end() {
        ws();
        return p_ == e_;
    }
    bool fail(const std::string& m) {
        if (error.empty()) error = m + " at header byte " + std::to_string(pos());
        return false;
    }
    size_t pos() const { return static_cast<size_t>(p_ - start_); }
    void set_start(const char* s) { start_ = s; }

    bool string(std::string& out) {
        out.clear();
        if (!take('"')) return false;
        while (p_ < e_ && *p_ != '"') {
            const unsigned char c = static_cast<unsigned char>(*p_++);
            if (c < 0x20) return fail("control character in string");
            if (c != '\\') {
                out.push_back(static_cast<char>(c));
                continue;
            }
            if (p_ >= e_) break;
            const char x = *p_++;
            switch (x) {
                case '"': out.push_back('"'); break;
                case '\\': out.push_back('\\'); break;
                case '/': out.push_back('/'); break;
                case 'b': out.push_back('\b'); break;
                case 'f': out.push_back('\f'); break;
                case 'n': out.push_back('\n'); break;
                case 'r': out.push_back('\r'); break;
                case 't': out.push_back('\t'); break;
                case 'u': {
                    uint32_t cp;
                    if (!hex4(cp)) return false;
                    if (cp >= 0xD800 && cp < 0xDC00) {  // high surrogate: a low one must follow
                        uint32_t lo;
                        if (e_ - p_ < 2 || p_[0] != '\\' || p_[1] != 'u') return fail("lone surrogate");
                        p_ += 2;
                        if (!hex4(lo)) return false;
                        if (lo < 0xDC00 || lo >= 0xE000) return fail("bad surrogate pair");
                        cp = 0x10000 + ((cp - 0xD800) << 10) + (lo - 0xDC00);
                    } else if (cp >= 0xDC00 && cp < 0xE000) {
                        return fail("lone surrogate");
                    }
                    utf8(cp, out);
                    break;
                }
                default: return fail("bad escape");
            }
        }
        if (p_ >= e_) return fail("unterminated string");
        ++p_;
        return true;
    }

    bool uint(uint64_t& v) {
        ws();
        if (p_ >= e_ || *p_ < '0' || *p_ > '9') return fail("expected a non-negative integer");
        v = 0;
        while (p_ < e_ && *p_ >= '0' && *p_ <= '9') {
            const uint64_t d = static_cast<uint64_t>(*p_ - '0');
            if (v > (UINT64_MAX - d) / 10) return fail("integer overflow");
            v = v * 10 + d;
            ++p_;
        }
        if (p_ < e_ && (*p_ == '.' || *p_ == 'e' || *p_ == 'E')) return fail("expected an integer");
        return true;
    }

    bool uint_array(std::vector<uint64_t>& out) {
        out.clear();
        if (!take('[')) return false;
        if (peek(']')) {
            ++p_;
            return true;
        }
        for (;;) {
            uint64_t v;
            if (!uint(v)) return false;
            out.push_back(v);
            if (peek(',')) {
                ++p_;
                continue;
            }
            return take(']');
        }
    }

    // Skips any JSON value (depth-limited).
    bool skip(int depth = 0) {
        if (depth > 64) return fail("nesting too deep");
        ws();
        if (p_ >= e_) return fail("unexpected end");
        const char c = *p_;
        if (c == '"') {
            std::string s;
            return string(s);
        }
        if (c == '{' || c == '[') {
            const char close = c == '{' ? '}' : ']';
            ++p_;
            if (peek(close)) {
                ++p_;
                return true;
            }
            for (;;) {
                if (c == '{') {
                    std::string k;
                    if (!string(k) || !take(':')) return false;
                }
                if (!skip(depth + 1)) return false;
                if (peek(',')) {
                    ++p_;
                    continue;
                }
                return take(close);
            }
        }
        for (const char* lit : {"true", "false", "null"}) {
            const size_t n = std::strlen(lit);
            if (static_cast<size_t>(e_ - p_) >= n && std::memcmp(p_, lit, n) == 0) {
                p_ += n;
                return true;
            }
        }
        if (c == '-' || (c >= '0' && c <= '9')) {
            ++p_;
            while (p_ < e_ && *p_ != '\0' && std::strchr("0123456789.eE+-", *p_) != nullptr) ++p_;
            return true;
        }
        return fail("unexpected character");
    }

private:
    bool hex4(uint32_t& v) {
        if (e_ - p_ < 4) return fail("short \\u escape");
        v = 0;
        for (int i = 0; i < 4; ++i) {
            const char h = *p_++;
            v <<= 4;
            if (h >= '0' && h <= '9') v |= static_cast<uint32_t>(h - '0');
            else if (h >= 'a' && h <= 'f') v |= static_cast<uint32_t>(h - 'a' + 10);
            else if (h >= 'A' && h <= 'F') v |= static_cast<uint32_t>(h - 'A' + 10);
            else return fail("bad \\u escape");
        }
        return true;
    }
    static void utf8(uint32_t cp, std::string& out) {
        if (cp < 0x80) {
            out.push_back(static_cast<char>(cp));
        } else if (cp < 0x800) {
            out.push_back(static_cast<char>(0xC0 | (cp >> 6)));
            out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
        } else if (cp < 0x10000) {
            out.push_back(static_cast<char>(0xE0 | (cp >> 12)));
            out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
            out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
        } else {
            out.push_back(static_cast<char>(0xF0 | (cp >> 18)));
            out.push_back(static_cast<char>(0x80 | ((cp >> 12) & 0x3F)));
            out.push_back(static_cast<char>(0x80 | ((cp >> 6) & 0x3F)));
            out.push_back(static_cast<char>(0x80 | (cp & 0x3F)));
        }
    }
    const char* p_;
    const char* e_;
    const char* start_ = nullptr;
};

constexpr uint64_t kMaxHeader = 100000000ull;  // the format's own limit on the JSON header

// Copies out of the mapping into pinned staging with several host threads: one thread
// moves about 10 GB/s out of the page cache, below what a host->device copy sustains
// (measured on the B200 hosts: 8 threads 16 GB/s end to end; pread from 16 threads 12).
void parallel_memcpy(uint8_t* dst, const uint8_t* src, uint64_t n) {
    constexpr uint64_t kPiece = 4u << 20;
    const unsigned hw = std::thread::hardware_concurrency();
    const unsigned nt = static_cast<unsigned>(std::max<uint64_t>(1, std::min<uint64_t>(std::min(hw ? hw : 1u, 8u), n / kPiece)));
    if (nt == 1) {
        std::memcpy(dst, src, n);
        return;
    }
    const uint64_t per = (n + nt - 1) / nt;
    std::vector<std::thread> th;
    th.reserve(nt - 1);
    for (unsigned t = 1; t < nt; ++t) {
        const uint64_t b = t * per, e = std::min<uint64_t>(n, b + per);
        if (b < e) th.emplace_back([=] { std::memcpy(dst + b, src + b, e - b); });
    }
    std::memcpy(dst, src, std::min<uint64_t>(n, per));
    for (std::thread& t : th) t.join();
}

}  // namespace

struct q38_st_file {
    int fd = -1;
    void* map = nullptr;
    size_t size = 0;
    const uint8_t* data = nullptr;  // start of the byte buffer
    uint64_t data_len = 0;
    std::vector<StTensor> tensors;  // header order
    std::vector<std::pair<std::string, std::string>> metadata;
    std::unordered_map<std::string, int64_t> index;
    ~q38_st_file() {
        if (map && map != MAP_FAILED) munmap(map, size);
        if (fd >= 0) close(fd);
    }
};

namespace {

bool parse_header(q38_st_file* f, const char* h, size_t n, std::string& err) {
    Json j(h, h + n);
    j.set_start(h);
    if (!j.take('{')) return err = j.error, false;
    if (j.peek('}')) {
        j.take('}');
    } else {
        for (;;) {
            std::string key;
            if (!j.string(key) || !j.take(':')) return err = j.error, false;
            if (key == "__metadata__") {
                if (!j.take('{')) return err = j.error, false;
                if (j.peek('}')) {
                    j.take('}');
                } else {
                    for (;;) {
                        std::string k, v;
                        if (!j.string(k) || !j.take(':') || !j.string(v)) return err = j.error, false;
                        f->metadata.emplace_back(std::move(k), std::move(v));
                        if (j.peek(',')) {
                            j.take(',');
                            continue;
                        }
                        if (!j.take('}')) return err = j.error, false;
                        break;
                    }
                }
            } else {
                StTensor t;
                t.name = key;
                bool has_dtype = false, has_shape = false, has_off = false;
                if (!j.take('{')) return err = j.error, false;
                if (!j.peek('}')) {
                    for (;;) {
                        std::string k;
                        if (!j.string(k) || !j.take(':')) return err = j.error, false;
                        if (k == "dtype") {
                            if (!j.string(t.dtype)) return err = j.error, false;
                            has_dtype = true;
                        } else if (k == "shape") {
                            std::vector<uint64_t> s;
                            if (!j.uint_array(s)) return err = j.error, false;
                            for (uint64_t d : s) {
                                if (d > static_cast<uint64_t>(INT64_MAX)) return err = "shape too large", false;
                                t.shape.push_back(static_cast<int64_t>(d));
                            }
                            has_shape = true;
                        } else if (k == "data_offsets") {
                            std::vector<uint64_t> o;
                            if (!j.uint_array(o)) return err = j.error, false;
                            if (o.size() != 2) return err = "tensor '" + key + "': data_offsets needs two entries", false;
                            t.begin = o[0];
                            t.end = o[1];
                            has_off = true;
                        } else if (!j.skip()) {
                            return err = j.error, false;
                        }
                        if (j.peek(',')) {
                            j.take(',');
                            continue;
                        }
                        break;
                    }
                }
                if (!j.take('}')) return err = j.error, false;
                if (!has_dtype || !has_shape || !has_off)
                    return err = "tensor '" + key + "' lacks dtype, shape or data_offsets", false;
                if (f->index.count(key)) return err = "duplicate tensor '" + key + "'", false;
                f->index.emplace(key, static_cast<int64_t>(f->tensors.size()));
                f->tensors.push_back(std::move(t));
            }
            if (j.peek(',')) {
                j.take(',');
                continue;
            }
            if (!j.take('}')) return err = j.error, false;
            break;
        }
    }
    if (!j.at_end()) return err = "trailing bytes after the header object", false;
    return true;
}

bool validate(q38_st_file* f, std::string& err) {
    std::vector<const StTensor*> byoff;
    byoff.reserve(f->tensors.size());
    for (const StTensor& t : f->tensors) {
        const int es = dtype_size(t.dtype);
        if (!es) return err = "tensor '" + t.name + "': unknown dtype " + t.dtype, false;
        if (t.shape.size() > 8) return err = "tensor '" + t.name + "': more than 8 dimensions", false;
        unsigned __int128 n = static_cast<unsigned>(es);
        for (int64_t d : t.shape) {
            n *= static_cast<uint64_t>(d);
            if (n > (static_cast<unsigned __int128>(1) << 63)) return err = "tensor '" + t.name + "': too large", false;
        }
        if (t.end < t.begin || static_cast<unsigned __int128>(t.end - t.begin) != n)
            return err = "tensor '" + t.name + "': data_offsets disagree with dtype and shape", false;
        byoff.push_back(&t);
    }
    std::sort(byoff.begin(), byoff.end(), [](const StTensor* a, const StTensor* b) {
        return a->begin != b->begin ? a->begin < b->begin : a->end < b->end;
    });
    uint64_t at = 0;
    for (const StTensor* t : byoff) {
        if (t->begin != at)
            return err = "tensor '" + t->name + "': data_offsets leave a gap or overlap another tensor", false;
        at = t->end;
    }
    if (at != f->data_len) return err = "the tensors do not cover the byte buffer exactly", false;
    return true;
}

q38_status open_error(const std::string& m) {
    g_open_error = m;
    return Q38_ERR_INVALID_ARGUMENT;
}

}  // namespace

extern "C" {

q38_status q38_st_open(const char* path, q38_st_file** out) {
    if (!path || !out) return open_error("null argument");
    *out = nullptr;
    g_open_error.clear();
    std::unique_ptr<q38_st_file> f(new q38_st_file);
    f->fd = open(path, O_RDONLY | O_CLOEXEC);
    if (f->fd < 0) return open_error(std::string("cannot open ") + path + ": " + std::strerror(errno));
    struct stat sb;
    if (fstat(f->fd, &sb) != 0) return open_error(std::string("cannot stat ") + path);
    f->size = static_cast<size_t>(sb.st_size);
    if (f->size < 8) return open_error("file shorter than the 8-byte header length");
    f->map = mmap(nullptr, f->size, PROT_READ, MAP_PRIVATE, f->fd, 0);
    if (f->map == MAP_FAILED) return open_error(std::string("cannot map ") + path + ": " + std::strerror(errno));
    const uint8_t* base = static_cast<const uint8_t*>(f->map);
    uint64_t n = 0;
    for (int i = 7; i >= 0; --i) n = (n << 8) | base[i];  // little-endian
    if (n > kMaxHeader) return open_error("header length above the format's limit");
    if (n > f->size - 8) return open_error("header length beyond the end of the file");
    f->data = base + 8 + n;
    f->data_len = f->size - 8 - n;
    std::string err;
    if (!parse_header(f.get(), reinterpret_cast<const char*>(base + 8), static_cast<size_t>(n), err) ||
        !validate(f.get(), err))
        return open_error(err);
    *out = f.release();
    return Q38_OK;
}

const char* q38_st_open_error(void) { return g_open_error.c_str(); }

void q38_st_close(q38_st_file* f) { delete f; }

int64_t q38_st_count(const q38_st_file* f) { return f ? static_cast<int64_t>(f->tensors.size()) : -1; }

int64_t q38_st_find(const q38_st_file* f, const char* name) {
    if (!f || !name) return -1;
    const auto it = f->index.find(name);
    return it == f->index.end() ? -1 : it->second;
}

q38_status q38_st_info(const q38_st_file* f, int64_t i, const char** name, const char** dtype, int* ndim,
                       int64_t* shape, uint64_t* nbytes) {
    if (!f || i < 0 || i >= static_cast<int64_t>(f->tensors.size())) return Q38_ERR_INVALID_ARGUMENT;
    const StTensor& t = f->tensors[static_cast<size_t>(i)];
    if (name) *name = t.name.c_str();
    if (dtype) *dtype = t.dtype.c_str();
    if (ndim) *ndim = static_cast<int>(t.shape.size());
    if (shape)
        for (size_t d = 0; d < t.shape.size(); ++d) shape[d] = t.shape[d];
    if (nbytes) *nbytes = t.end - t.begin;
    return Q38_OK;
}

const void* q38_st_data(const q38_st_file* f, int64_t i) {
    if (!f || i < 0 || i >= static_cast<int64_t>(f->tensors.size())) return nullptr;
    return f->data + f->tensors[static_cast<size_t>(i)].begin;
}

int64_t q38_st_metadata_count(const q38_st_file* f) { return f ? static_cast<int64_t>(f->metadata.size()) : -1; }

q38_status q38_st_metadata_entry(const q38_st_file* f, int64_t i, const char** key, const char** value) {
    if (!f || i < 0 || i >= static_cast<int64_t>(f->metadata.size())) return Q38_ERR_INVALID_ARGUMENT;
    if (key) *key = f->metadata[static_cast<size_t>(i)].first.c_str();
    if (value) *value = f->metadata[static_cast<size_t>(i)].second.c_str();
    return Q38_OK;
}

q38_status q38_st_copy_block_to_device(q38_ctx* ctx, const q38_st_file* f, int64_t i, uint64_t row_bytes,
                                       uint64_t row0, uint64_t rows, uint64_t col_byte0, uint64_t col_bytes,
                                       void* dst, uint64_t dst_pitch) {
    using namespace q38;
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    if (!f || i < 0 || i >= static_cast<int64_t>(f->tensors.size()) || !dst)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "st_copy_block_to_device: bad file, index or destination");
    const StTensor& t = f->tensors[static_cast<size_t>(i)];
    const uint64_t nbytes = t.end - t.begin;
    if (row_bytes == 0 || nbytes % row_bytes || col_bytes == 0 || col_byte0 > row_bytes ||
        col_bytes > row_bytes - col_byte0 || row0 > nbytes / row_bytes || rows > nbytes / row_bytes - row0 ||
        dst_pitch < col_bytes)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT,
                    "st_copy_block_to_device: block outside tensor '%s' (%llu bytes)", t.name.c_str(),
                    static_cast<unsigned long long>(nbytes));
    if (rows == 0) return Q38_OK;
    if (cudaSetDevice(ctx->device) != cudaSuccess) return check_launch(ctx, "cudaSetDevice");
    constexpr size_t kHalf = 32u << 20;
    if (!ctx->host_stage) {
        for (cudaEvent_t& e : ctx->stage_done)
            if (!e && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess)
                return check_launch(ctx, "st_copy_block_to_device: event creation");
        if (cudaHostAlloc(&ctx->host_stage, 2 * kHalf, cudaHostAllocDefault) != cudaSuccess) {
            ctx->host_stage = nullptr;
            cudaGetLastError();
            return fail(ctx, Q38_ERR_OUT_OF_MEMORY, "st_copy_block_to_device: pinned staging allocation failed");
        }
        ctx->host_stage_bytes = kHalf;
    }
    const uint64_t H = ctx->host_stage_bytes;
    const uint8_t* src = f->data + t.begin + row0 * row_bytes + col_byte0;
    uint8_t* d = static_cast<uint8_t*>(dst);
    int half = 0;
    // the next free staging half (its previous copy has completed)
    auto acquire = [&](uint8_t** stage) {
        *stage = static_cast<uint8_t*>(ctx->host_stage) + half * H;
        return cudaEventSynchronize(ctx->stage_done[half]);
    };
    // marks the half in use by the copy just enqueued and moves to the other half
    auto release = [&](cudaError_t e) {
        if (e == cudaSuccess) e = cudaEventRecord(ctx->stage_done[half], ctx->stream);
        half ^= 1;
        return e;
    };
    cudaError_t e = cudaSuccess;
    uint8_t* stage = nullptr;
    if (col_bytes == row_bytes && dst_pitch == row_bytes) {
        // whole rows: one contiguous byte range
        const uint64_t total = rows * row_bytes;
        for (uint64_t off = 0; off < total && e == cudaSuccess; off += H) {
            const uint64_t n = std::min<uint64_t>(H, total - off);
            if ((e = acquire(&stage)) != cudaSuccess) break;
            parallel_memcpy(stage, src + off, n);
            e = release(cudaMemcpyAsync(d + off, stage, n, cudaMemcpyHostToDevice, ctx->stream));
        }
    } else if (col_bytes <= H) {
        // a column range of each row: rows gathered densely, then one 2-D copy per half
        const uint64_t per = H / col_bytes;
        for (uint64_t r = 0; r < rows && e == cudaSuccess; r += per) {
            const uint64_t nr = std::min<uint64_t>(per, rows - r);
            if ((e = acquire(&stage)) != cudaSuccess) break;
            for (uint64_t k = 0; k < nr; ++k) std::memcpy(stage + k * col_bytes, src + (r + k) * row_bytes, col_bytes);
            e = release(cudaMemcpy2DAsync(d + r * dst_pitch, dst_pitch, stage, col_bytes, col_bytes, nr,
                                          cudaMemcpyHostToDevice, ctx->stream));
        }
    } else {
        // column ranges wider than a half: each row in pieces
        for (uint64_t r = 0; r < rows && e == cudaSuccess; ++r)
            for (uint64_t off = 0; off < col_bytes && e == cudaSuccess; off += H) {
                const uint64_t n = std::min<uint64_t>(H, col_bytes - off);
                if ((e = acquire(&stage)) != cudaSuccess) break;
                parallel_memcpy(stage, src + r * row_bytes + off, n);
                e = release(cudaMemcpyAsync(d + r * dst_pitch + off, stage, n, cudaMemcpyHostToDevice, ctx->stream));
            }
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(ctx, Q38_ERR_CUDA, "st_copy_block_to_device: copy failed: %s", cudaGetErrorString(e));
    }
    // the staging halves are reused by the next call; the copies themselves stay ordered
    // on the context's stream
    return Q38_OK;
}

q38_status q38_st_copy_to_device(q38_ctx* ctx, const q38_st_file* f, int64_t i, void* dst, uint64_t dst_bytes) {
    using namespace q38;
    if (!ctx) return Q38_ERR_INVALID_ARGUMENT;
    if (!f || i < 0 || i >= static_cast<int64_t>(f->tensors.size()))
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "st_copy_to_device: bad file or index");
    const StTensor& t = f->tensors[static_cast<size_t>(i)];
    const uint64_t nbytes = t.end - t.begin;
    if (dst_bytes < nbytes)
        return fail(ctx, Q38_ERR_INVALID_ARGUMENT, "st_copy_to_device: tensor '%s' needs %llu bytes, buffer has %llu",
                    t.name.c_str(), static_cast<unsigned long long>(nbytes),
                    static_cast<unsigned long long>(dst_bytes));
    if (nbytes == 0) return Q38_OK;
    return q38_st_copy_block_to_device(ctx, f, i, nbytes, 0, 1, 0, nbytes, dst, nbytes);
}

}  // extern "C"
