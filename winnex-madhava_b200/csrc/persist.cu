// Index files: save a built index, load it back without sorting again.
//
// Replaces MadhavaL2::save_index / load_index (src/winnex_madhava.cpp:1111-1217).
// The reference file holds the bound engine's projections and norms and leaves
// the corpus out (the caller re-attaches it).  Here the search state IS the
// norm-sorted corpus, so the file holds each shard's full level exactly as the
// scan reads it: u8 rows with their padded stride, |v|^2 and global row ids
// (float corpora: float rows, float norms, ids).  Everything else is derived
// on load: the nested sample levels pick rows by a hash of the row id, so they
// come out the same, and the TMA maps follow from the buffers.
//
// I/O streams through pinned staging buffers in groups of eight chunks: the
// chunks of one group are read from (or written to) the file by parallel host
// threads while the previous group crosses PCIe.  A loaded shard is
// checked on its GPU before it is used: every row's |v|^2 is recomputed and
// compared with the stored one, the (norm, id) order must ascend strictly and
// ids must lie in the shard's range, so a damaged or foreign file fails the
// load instead of returning wrong neighbours.
//
// The layout is written out in include/winnex_madhava_b200.h.
#include <errno.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <memory>
#include <exception>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

#include "internal.h"

namespace mdh {
namespace {

constexpr char kMagic[8] = {'M', 'D', 'H', 'B', '2', '0', '0', 'I'};
constexpr uint32_t kVersion = 1;
constexpr uint64_t kHeaderBytes = 64;
constexpr uint64_t kShardEntryBytes = 32;
constexpr uint64_t kAlign = 4096;
constexpr int32_t kMaxShards = 4096;
constexpr size_t kStageBytes = size_t(8) << 20;  // per staging buffer
constexpr int kIoLanes = 8;                        // chunks read or written in parallel

struct FileShard {
    int64_t rows = 0;
    int64_t id_base = 0;
    uint64_t offset = 0;
    uint64_t bytes = 0;
};

struct FileHeader {
    uint32_t kind = 0;  // 0 u8 rows, 1 float32 rows
    int64_t n = 0;
    int32_t dim = 0;
    int32_t stride = 0;  // elements per stored row
    int32_t metric = 0;
    uint64_t data_offset = 0;
    uint64_t file_size = 0;
    std::vector<FileShard> shards;
};

uint64_t align_up(uint64_t a) { return (a + kAlign - 1) / kAlign * kAlign; }

uint64_t row_bytes(uint32_t kind, int32_t stride) {
    return (kind == 0 ? (uint64_t)stride : (uint64_t)stride * 4) + 8;  // row + norm + id
}

[[noreturn]] void io_fail(const std::string& path, const std::string& what) {
    throw Error(MDH_ERR_IO, "index file " + path + ": " + what);
}

struct Fd {
    int fd = -1;
    ~Fd() {
        if (fd >= 0) close(fd);
    }
};

void write_all(int fd, const void* buf, size_t len, uint64_t off, const std::string& path) {
    const char* p = static_cast<const char*>(buf);
    while (len > 0) {
        ssize_t w = pwrite(fd, p, len, (off_t)off);
        if (w < 0 && errno == EINTR) continue;
        if (w <= 0) io_fail(path, std::string("write failed: ") + (w < 0 ? strerror(errno) : "no progress"));
        p += w;
        len -= (size_t)w;
        off += (uint64_t)w;
    }
}

void read_all(int fd, void* buf, size_t len, uint64_t off, const std::string& path) {
    char* p = static_cast<char*>(buf);
    while (len > 0) {
        ssize_t r = pread(fd, p, len, (off_t)off);
        if (r < 0 && errno == EINTR) continue;
        if (r < 0) io_fail(path, std::string("read failed: ") + strerror(errno));
        if (r == 0) io_fail(path, "file is truncated");
        p += r;
        len -= (size_t)r;
        off += (uint64_t)r;
    }
}

template <class T>
void put(std::vector<uint8_t>& b, size_t at, T v) {
    std::memcpy(b.data() + at, &v, sizeof(T));
}
template <class T>
T get(const uint8_t* b, size_t at) {
    T v;
    std::memcpy(&v, b + at, sizeof(T));
    return v;
}

// Reads and validates the header and shard table against the file's size.
FileHeader read_header(int fd, const std::string& path) {
    struct stat stt;
    if (fstat(fd, &stt) != 0) io_fail(path, std::string("stat failed: ") + strerror(errno));
    const uint64_t actual = (uint64_t)stt.st_size;
    if (actual < kHeaderBytes) io_fail(path, "file is truncated (no header)");
    uint8_t h[kHeaderBytes];
    read_all(fd, h, sizeof(h), 0, path);
    if (std::memcmp(h, kMagic, 8) != 0) io_fail(path, "not an index file (bad magic)");
    if (get<uint32_t>(h, 8) != kVersion)
        io_fail(path, "unsupported version " + std::to_string(get<uint32_t>(h, 8)));
    FileHeader f;
    f.kind = get<uint32_t>(h, 12);
    f.n = get<int64_t>(h, 16);
    f.dim = get<int32_t>(h, 24);
    f.stride = get<int32_t>(h, 28);
    f.metric = get<int32_t>(h, 32);
    const int32_t nsh = get<int32_t>(h, 36);
    f.data_offset = get<uint64_t>(h, 40);
    f.file_size = get<uint64_t>(h, 48);
    if (f.kind > 1) io_fail(path, "unknown row kind " + std::to_string(f.kind));
    if (f.dim < 1 || f.dim > 4096) io_fail(path, "dim out of range");
    const int32_t want_stride = f.kind == 0 ? (int32_t)round_up(f.dim, kRowAlign) : f.dim;
    if (f.stride != want_stride) io_fail(path, "row stride does not match dim");
    if (f.metric != MDH_METRIC_COSINE && f.metric != MDH_METRIC_L2) io_fail(path, "unknown metric");
    if (nsh < 1 || nsh > kMaxShards) io_fail(path, "shard count out of range");
    if (f.n < 0 || f.n > 0x7FFFFFFF) io_fail(path, "row count out of range");
    if (f.file_size != actual)
        io_fail(path, f.file_size > actual ? "file is truncated" : "file is longer than its header says");
    const uint64_t table_end = kHeaderBytes + kShardEntryBytes * (uint64_t)nsh;
    if (f.data_offset % kAlign != 0 || f.data_offset < table_end || f.data_offset > actual)
        io_fail(path, "bad data offset");
    std::vector<uint8_t> t((size_t)(kShardEntryBytes * nsh));
    read_all(fd, t.data(), t.size(), kHeaderBytes, path);
    uint64_t prev_end = f.data_offset;
    int64_t total = 0;
    const uint64_t per_row = row_bytes(f.kind, f.stride);
    for (int32_t i = 0; i < nsh; i++) {
        FileShard s;
        const uint8_t* e = t.data() + kShardEntryBytes * i;
        s.rows = get<int64_t>(e, 0);
        s.id_base = get<int64_t>(e, 8);
        s.offset = get<uint64_t>(e, 16);
        s.bytes = get<uint64_t>(e, 24);
        const std::string which = "shard " + std::to_string(i) + ": ";
        if (s.rows < 0 || s.rows > f.n) io_fail(path, which + "row count out of range");
        if (s.id_base < 0 || s.id_base + s.rows > 0x7FFFFFFF) io_fail(path, which + "row ids out of int32 range");
        // The shards' id ranges tile one run [first id, first id + n) in file
        // order, so no two shards can hand out the same id.
        if (i > 0 && s.id_base != f.shards.back().id_base + f.shards.back().rows)
            io_fail(path, which + "id range does not follow the previous shard's");
        if (s.bytes != (uint64_t)s.rows * per_row) io_fail(path, which + "size does not match its row count");
        if (s.offset % kAlign != 0 || s.offset < prev_end) io_fail(path, which + "bad offset");
        if (s.offset > actual || s.bytes > actual - s.offset) io_fail(path, which + "runs past the end of the file");
        prev_end = s.offset + s.bytes;
        total += s.rows;
        f.shards.push_back(s);
    }
    if (total != f.n) io_fail(path, "shard row counts do not add up to n");
    return f;
}

// Pinned staging for the file <-> device pipelines: two halves of kIoLanes
// chunk buffers each, and one copy event per half.  A group of up to kIoLanes
// chunks is read (or written) by parallel host threads in one half while the
// other half's copies run on the stream.  The buffers are portable (pinned
// for every device); the events belong to one device, so use_device() makes
// them anew on the current device before each shard's copies.
struct Staging {
    static constexpr int kSlots = 2 * kIoLanes;
    uint8_t* buf[kSlots] = {};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    Staging() {
        for (int i = 0; i < kSlots; i++) {
            void* p = nullptr;
            cudaError_t e = cudaHostAlloc(&p, kStageBytes, cudaHostAllocPortable);
            if (e != cudaSuccess) {
                cudaGetLastError();
                release();
                throw Error(MDH_ERR_OOM, std::string("pinned staging allocation failed: ") + cudaGetErrorString(e));
            }
            buf[i] = static_cast<uint8_t*>(p);
        }
    }
    // Waits for the last copies of each half (an error can leave some in
    // flight), then drops the events.
    void drop_events() {
        for (int i = 0; i < 2; i++) {
            if (ev[i]) cudaEventSynchronize(ev[i]);
            if (ev[i]) cudaEventDestroy(ev[i]);
            ev[i] = nullptr;
        }
    }
    void use_device() {
        drop_events();
        for (int i = 0; i < 2; i++) {
            cudaError_t e = cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming);
            if (e != cudaSuccess) {
                cudaGetLastError();
                throw_cuda(e, "cudaEventCreateWithFlags", __FILE__, __LINE__);
            }
        }
    }
    void release() {
        drop_events();
        for (int i = 0; i < kSlots; i++) {
            if (buf[i]) cudaFreeHost(buf[i]);
            buf[i] = nullptr;
        }
    }
    ~Staging() { release(); }
};

// Runs io(lane) for lanes [0, lanes) on parallel threads (lane 0 on the
// caller) and rethrows the first error after all have finished.
template <class F>
void parallel_lanes(int lanes, F&& io) {
    std::vector<std::exception_ptr> err((size_t)lanes);
    auto run = [&](int t) {
        try {
            io(t);
        } catch (...) {
            err[(size_t)t] = std::current_exception();
        }
    };
    std::vector<std::thread> th;
    for (int t = 1; t < lanes; t++) th.emplace_back(run, t);
    run(0);
    for (auto& x : th) x.join();
    for (auto& e : err)
        if (e) std::rethrow_exception(e);
}

// Device -> file.  Group g's chunks are copied into half g%2 while group
// g-1's chunks are written from the other half.
void device_to_file(int fd, uint64_t off, const void* dev, uint64_t bytes, cudaStream_t st, Staging& sg,
                    const std::string& path) {
    const uint64_t nchunks = (bytes + kStageBytes - 1) / kStageBytes;
    const uint64_t groups = (nchunks + kIoLanes - 1) / kIoLanes;
    auto len_of = [&](uint64_t c) { return (size_t)std::min<uint64_t>(kStageBytes, bytes - c * kStageBytes); };
    for (uint64_t g = 0; g <= groups; g++) {
        if (g < groups) {
            const int half = (int)(g & 1);
            for (int t = 0; t < kIoLanes; t++) {
                const uint64_t c = g * kIoLanes + t;
                if (c >= nchunks) break;
                MDH_CUDA(cudaMemcpyAsync(sg.buf[half * kIoLanes + t], static_cast<const uint8_t*>(dev) + c * kStageBytes,
                                         len_of(c), cudaMemcpyDeviceToHost, st));
            }
            MDH_CUDA(cudaEventRecord(sg.ev[half], st));
        }
        if (g > 0) {
            const uint64_t p = g - 1;
            const int half = (int)(p & 1);
            MDH_CUDA(cudaEventSynchronize(sg.ev[half]));
            const int lanes = (int)std::min<uint64_t>(kIoLanes, nchunks - p * kIoLanes);
            parallel_lanes(lanes, [&](int t) {
                const uint64_t c = p * kIoLanes + t;
                write_all(fd, sg.buf[half * kIoLanes + t], len_of(c), off + c * kStageBytes, path);
            });
        }
    }
}

// File -> device.  Group g's chunks are read into half g%2 (after group g-2's
// copies have left it) while group g-1's copies run.
void file_to_device(int fd, uint64_t off, void* dev, uint64_t bytes, cudaStream_t st, Staging& sg,
                    const std::string& path) {
    const uint64_t nchunks = (bytes + kStageBytes - 1) / kStageBytes;
    const uint64_t groups = (nchunks + kIoLanes - 1) / kIoLanes;
    auto len_of = [&](uint64_t c) { return (size_t)std::min<uint64_t>(kStageBytes, bytes - c * kStageBytes); };
    for (uint64_t g = 0; g < groups; g++) {
        const int half = (int)(g & 1);
        if (g >= 2) MDH_CUDA(cudaEventSynchronize(sg.ev[half]));
        const int lanes = (int)std::min<uint64_t>(kIoLanes, nchunks - g * kIoLanes);
        parallel_lanes(lanes, [&](int t) {
            const uint64_t c = g * kIoLanes + t;
            read_all(fd, sg.buf[half * kIoLanes + t], len_of(c), off + c * kStageBytes, path);
        });
        for (int t = 0; t < lanes; t++) {
            const uint64_t c = g * kIoLanes + t;
            MDH_CUDA(cudaMemcpyAsync(static_cast<uint8_t*>(dev) + c * kStageBytes, sg.buf[half * kIoLanes + t],
                                     len_of(c), cudaMemcpyHostToDevice, st));
        }
        MDH_CUDA(cudaEventRecord(sg.ev[half], st));
    }
    MDH_CUDA(cudaStreamSynchronize(st));
}

// u8 level check, 8 lanes per row (16 bytes each per step): the row's |v|^2
// over its padded stride equals the stored norm, its id lies in [id_lo,
// id_hi), and (norm, id) ascends strictly from the previous position.
// seen: a zeroed bitmap of id_hi - id_lo bits; each id sets its bit, and an
// id whose bit was already set is a duplicate.  n ids in range with no
// duplicate are a permutation of [id_lo, id_hi).
__global__ void k_check_level_u8(const uint8_t* __restrict__ rows, const int32_t* __restrict__ norms,
                                 const int32_t* __restrict__ ids, int64_t n, int dpad, int64_t id_lo, int64_t id_hi,
                                 uint32_t* __restrict__ seen, unsigned long long* __restrict__ bad) {
    const int64_t r = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 3;
    const int l8 = threadIdx.x & 7;
    uint32_t s = 0;
    if (r < n) {
        const uint8_t* row = rows + (size_t)r * dpad;
        for (int off = l8 * 16; off < dpad; off += 128) {
            uint4 v = *reinterpret_cast<const uint4*>(row + off);
            s = __dp4a(v.x, v.x, s);
            s = __dp4a(v.y, v.y, s);
            s = __dp4a(v.z, v.z, s);
            s = __dp4a(v.w, v.w, s);
        }
    }
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    if (r < n && l8 == 0) {
        const int32_t nr = norms[r], id = ids[r];
        bool ok = (int32_t)s == nr && id >= id_lo && id < id_hi;
        if (id >= id_lo && id < id_hi) {
            const int64_t b = id - id_lo;
            const uint32_t bit = 1u << (b & 31);
            if (atomicOr(seen + (b >> 5), bit) & bit) ok = false;
        }
        if (r > 0) {
            const int32_t np = norms[r - 1], ip = ids[r - 1];
            ok = ok && (np < nr || (np == nr && ip < id));
        }
        if (!ok) atomicAdd(bad, 1ull);
    }
}

// Float level check: float corpora keep id order (id = id_base + position);
// L2 norms are the sequential FMA chain the build used, cosine norms are 1.
__global__ void k_check_level_f32(const float* __restrict__ rows, const float* __restrict__ nf,
                                  const int32_t* __restrict__ ids, int64_t n, int dim, int cosine, int64_t id_base,
                                  unsigned long long* __restrict__ bad) {
    const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= n) return;
    bool ok = (int64_t)ids[r] == id_base + r;
    if (cosine) {
        ok = ok && nf[r] == 1.0f;
    } else {
        float s = 0.0f;
        const float* row = rows + (size_t)r * dim;
        for (int j = 0; j < dim; j++) s = __fmaf_rn(row[j], row[j], s);
        ok = ok && __float_as_uint(s) == __float_as_uint(nf[r]);
    }
    if (!ok) atomicAdd(bad, 1ull);
}

uint64_t check_level(const mdh_index* ix, const Shard& sh, const Level& lv) {
    if (lv.n == 0) return 0;
    unsigned long long* bad = nullptr;
    const size_t seen_bytes = ix->is_f32 ? 0 : (size_t)((sh.n + 31) / 32) * 4;
    MDH_CUDA(cudaMalloc(&bad, sizeof(unsigned long long) + seen_bytes));
    uint32_t* seen = reinterpret_cast<uint32_t*>(bad + 1);
    unsigned long long h = 0;
    try {
        MDH_CUDA(cudaMemsetAsync(bad, 0, sizeof(unsigned long long) + seen_bytes, sh.stream));
        if (ix->is_f32)
            k_check_level_f32<<<(unsigned)((lv.n + 255) / 256), 256, 0, sh.stream>>>(
                lv.rows_f32, lv.norms_f32, lv.ids, lv.n, ix->dim, ix->metric == MDH_METRIC_COSINE, sh.id_base, bad);
        else
            k_check_level_u8<<<(unsigned)((lv.n * 8 + 255) / 256), 256, 0, sh.stream>>>(
                lv.rows, lv.norms, lv.ids, lv.n, ix->dpad, sh.id_base, sh.id_base + sh.n, seen, bad);
        MDH_CUDA(cudaGetLastError());
        MDH_CUDA(cudaMemcpyAsync(&h, bad, sizeof(h), cudaMemcpyDeviceToHost, sh.stream));
        MDH_CUDA(cudaStreamSynchronize(sh.stream));
    } catch (...) {
        cudaFree(bad);
        throw;
    }
    cudaFree(bad);
    return h;
}

void save_impl(mdh_index* ix, const char* cpath) {
    MDH_REQUIRE(ix, MDH_ERR_INVALID_ARG, "null index");
    MDH_REQUIRE(cpath && *cpath, MDH_ERR_INVALID_ARG, "empty path");
    std::lock_guard<std::mutex> lock(ix->mu);
    const std::string path(cpath), tmp = path + ".tmp";
    const uint32_t kind = ix->is_f32 ? 1 : 0;
    const int32_t stride = ix->is_f32 ? ix->dim : ix->dpad;
    const int32_t nsh = (int32_t)ix->shards.size();
    MDH_REQUIRE(nsh >= 1 && nsh <= kMaxShards, MDH_ERR_INVALID_ARG, "index has no shards");
    const uint64_t per_row = row_bytes(kind, stride);
    const uint64_t data_off = align_up(kHeaderBytes + kShardEntryBytes * (uint64_t)nsh);
    std::vector<FileShard> table((size_t)nsh);
    uint64_t at = data_off;
    for (int32_t i = 0; i < nsh; i++) {
        const Shard& sh = ix->shards[(size_t)i];
        MDH_REQUIRE(!sh.levels.empty() && sh.levels.back().n == sh.n, MDH_ERR_INTERNAL, "shard has no full level");
        table[(size_t)i] = {sh.n, sh.id_base, at, (uint64_t)sh.n * per_row};
        at = align_up(at + table[(size_t)i].bytes);
    }
    uint64_t file_size = data_off;
    for (const FileShard& s : table) file_size = std::max(file_size, s.offset + s.bytes);

    std::vector<uint8_t> head((size_t)data_off, 0);
    std::memcpy(head.data(), kMagic, 8);
    put<uint32_t>(head, 8, kVersion);
    put<uint32_t>(head, 12, kind);
    put<int64_t>(head, 16, ix->n);
    put<int32_t>(head, 24, ix->dim);
    put<int32_t>(head, 28, stride);
    put<int32_t>(head, 32, ix->metric);
    put<int32_t>(head, 36, nsh);
    put<uint64_t>(head, 40, data_off);
    put<uint64_t>(head, 48, file_size);
    for (int32_t i = 0; i < nsh; i++) {
        const size_t e = (size_t)(kHeaderBytes + kShardEntryBytes * i);
        put<int64_t>(head, e, table[(size_t)i].rows);
        put<int64_t>(head, e + 8, table[(size_t)i].id_base);
        put<uint64_t>(head, e + 16, table[(size_t)i].offset);
        put<uint64_t>(head, e + 24, table[(size_t)i].bytes);
    }

    Fd f;
    f.fd = open(tmp.c_str(), O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644);
    if (f.fd < 0) io_fail(tmp, std::string("cannot create: ") + strerror(errno));
    try {
        write_all(f.fd, head.data(), head.size(), 0, tmp);
        Staging sg;
        for (int32_t i = 0; i < nsh; i++) {
            Shard& sh = ix->shards[(size_t)i];
            const Level& lv = sh.levels.back();
            MDH_CUDA(cudaSetDevice(sh.device));
            sg.use_device();
            const uint64_t n = (uint64_t)sh.n;
            const uint64_t rows_bytes = n * (kind == 0 ? (uint64_t)stride : (uint64_t)stride * 4);
            uint64_t off = table[(size_t)i].offset;
            if (kind == 0) {
                device_to_file(f.fd, off, lv.rows, rows_bytes, sh.stream, sg, tmp);
                device_to_file(f.fd, off + rows_bytes, lv.norms, n * 4, sh.stream, sg, tmp);
            } else {
                device_to_file(f.fd, off, lv.rows_f32, rows_bytes, sh.stream, sg, tmp);
                device_to_file(f.fd, off + rows_bytes, lv.norms_f32, n * 4, sh.stream, sg, tmp);
            }
            device_to_file(f.fd, off + rows_bytes + n * 4, lv.ids, n * 4, sh.stream, sg, tmp);
        }
        if (ftruncate(f.fd, (off_t)file_size) != 0) io_fail(tmp, std::string("truncate failed: ") + strerror(errno));
        if (fsync(f.fd) != 0) io_fail(tmp, std::string("fsync failed: ") + strerror(errno));
        close(f.fd);
        f.fd = -1;
        if (rename(tmp.c_str(), path.c_str()) != 0) io_fail(path, std::string("rename failed: ") + strerror(errno));
    } catch (...) {
        if (f.fd >= 0) {
            close(f.fd);
            f.fd = -1;
        }
        unlink(tmp.c_str());
        throw;
    }
}

void load_impl(const char* cpath, const int32_t* devices, int32_t ndev, mdh_index** out) {
    MDH_REQUIRE(out, MDH_ERR_INVALID_ARG, "null output pointer");
    *out = nullptr;
    MDH_REQUIRE(cpath && *cpath, MDH_ERR_INVALID_ARG, "empty path");
    const std::string path(cpath);
    Fd f;
    f.fd = open(cpath, O_RDONLY | O_CLOEXEC);
    if (f.fd < 0) io_fail(path, std::string("cannot open: ") + strerror(errno));
    const FileHeader h = read_header(f.fd, path);
    const int nsh = (int)h.shards.size();
    std::vector<int> devs;
    if (devices && ndev > 0) {
        MDH_REQUIRE(ndev == nsh, MDH_ERR_INVALID_ARG,
                    "devices must list one GPU per shard of the file (" + std::to_string(nsh) + ")");
        for (int i = 0; i < ndev; i++) devs.push_back(devices[i]);
    } else {
        int cur = 0;
        cudaError_t e = cudaGetDevice(&cur);
        if (e != cudaSuccess) {
            cudaGetLastError();
            throw Error(MDH_ERR_CUDA, "no CUDA device is available (this library has no CPU fallback)");
        }
        devs.assign((size_t)nsh, cur);
    }
    for (int d : devs) check_device_usable(d);

    std::unique_ptr<mdh_index> ix(new mdh_index());
    ix->n = h.n;
    ix->dim = h.dim;
    ix->dpad = (int)round_up(h.dim, kRowAlign);
    ix->metric = h.metric;
    ix->is_f32 = h.kind == 1;
    ix->shards.resize((size_t)nsh);
    const bool u8 = !ix->is_f32;
    try {
        Staging sg;
        for (int i = 0; i < nsh; i++) {
            Shard& sh = ix->shards[(size_t)i];
            const FileShard& fs = h.shards[(size_t)i];
            sh.device = devs[(size_t)i];
            MDH_CUDA(cudaSetDevice(sh.device));
            sg.use_device();
            MDH_CUDA(cudaStreamCreateWithFlags(&sh.stream, cudaStreamNonBlocking));
            sh.n = fs.rows;
            sh.id_base = fs.id_base;
            Level full;
            sh.levels.push_back(full);
            Level& lv = sh.levels.back();
            alloc_level(lv, fs.rows, ix->dpad, ix->dim, u8, !u8, sh.stream);
            const uint64_t n = (uint64_t)fs.rows;
            const uint64_t rows_bytes = n * (u8 ? (uint64_t)h.stride : (uint64_t)h.stride * 4);
            if (u8) {
                file_to_device(f.fd, fs.offset, lv.rows, rows_bytes, sh.stream, sg, path);
                file_to_device(f.fd, fs.offset + rows_bytes, lv.norms, n * 4, sh.stream, sg, path);
            } else {
                file_to_device(f.fd, fs.offset, lv.rows_f32, rows_bytes, sh.stream, sg, path);
                file_to_device(f.fd, fs.offset + rows_bytes, lv.norms_f32, n * 4, sh.stream, sg, path);
            }
            file_to_device(f.fd, fs.offset + rows_bytes + n * 4, lv.ids, n * 4, sh.stream, sg, path);
            const uint64_t bad = check_level(ix.get(), sh, lv);
            if (bad) io_fail(path, "shard " + std::to_string(i) + ": " + std::to_string(bad) +
                                       " rows fail the integrity check (norm, order or id range)");
            finish_shard(ix.get(), sh, u8, !u8);
        }
    } catch (...) {
        for (auto& sh : ix->shards) free_shard(sh);
        throw;
    }
    *out = ix.release();
}

template <class F>
mdh_status guarded(F&& fn) {
    using Fn = std::remove_reference_t<F>;
    return run_guarded([](void* c) { (*static_cast<Fn*>(c))(); }, const_cast<void*>(static_cast<const void*>(&fn)));
}

}  // namespace
}  // namespace mdh

using namespace mdh;

extern "C" {

mdh_status mdh_index_save(mdh_index* index, const char* path) {
    return guarded([&] { save_impl(index, path); });
}

mdh_status mdh_index_load(const char* path, const int32_t* devices, int32_t ndev, mdh_index** out) {
    return guarded([&] { load_impl(path, devices, ndev, out); });
}

mdh_status mdh_index_file_info(const char* path, int64_t* n, int32_t* dim, int32_t* metric, int32_t* shards,
                               int32_t* is_float) {
    return guarded([&] {
        MDH_REQUIRE(path && *path, MDH_ERR_INVALID_ARG, "empty path");
        Fd f;
        f.fd = open(path, O_RDONLY | O_CLOEXEC);
        if (f.fd < 0) io_fail(path, std::string("cannot open: ") + strerror(errno));
        const FileHeader h = read_header(f.fd, path);
        if (n) *n = h.n;
        if (dim) *dim = h.dim;
        if (metric) *metric = h.metric;
        if (shards) *shards = (int32_t)h.shards.size();
        if (is_float) *is_float = (int32_t)h.kind;
    });
}

}  // extern "C"
