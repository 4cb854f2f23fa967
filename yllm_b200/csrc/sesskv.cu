// sesskv.cu -- the engine's session KV file, written from and read into device
// memory.
//
// Reference: sess_kv_save / sess_kv_load (cache.c:174-195, 219-247) write and
// read the host KV blob of the CPU engine: an 8-byte magic ("YLLMSKV0", the
// first 8 bytes of SESS_KV_MAGIC, cache.c:129), then n_blocks, kv_dim,
// max_seq and pos as uint32, then for every block l = 1..n_blocks the first
// pos rows of K region l and of V region n_blocks + l of the
// (2*n_blocks + 1)-region blob (engine.c:261).  A load checks the magic and
// that n_blocks, kv_dim and max_seq equal the engine's and pos <= max_seq.
//
// Here the blob lives in HBM.  The file is cut into chunks at known offsets,
// and host threads move them through pinned staging buffers, two per thread:
// one chunk's device copy runs while the previous one is written with pwrite
// or read with pread.  A load spreads the chunks over kWorkers readers, since
// a single thread cannot copy out of the page cache at memory speed; a save
// has one writer, since writes to one file serialise in the kernel anyway.
#include "common.cuh"

#include <stdio.h>

#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace yattn {
namespace {

constexpr char kMagic[8] = {'Y', 'L', 'L', 'M', 'S', 'K', 'V', '0'};
constexpr size_t kChunk = size_t(16) << 20;   // bytes per staging buffer
constexpr int kWorkers = 4;                    // host threads moving chunks
constexpr size_t kHeader = 24;                 // magic + four uint32

struct Span {
    size_t off;     // element offset in the blob
    size_t bytes;
};

// The file's row spans in file order (cache.c:187-193).
std::vector<Span> spans_of(uint32_t nb, uint32_t kv_dim, uint32_t max_seq, uint32_t pos) {
    std::vector<Span> s;
    const size_t region = static_cast<size_t>(max_seq) * kv_dim;
    const size_t bytes = static_cast<size_t>(pos) * kv_dim * 2;
    if (bytes == 0) return s;
    for (uint32_t l = 1; l <= nb; ++l) {
        s.push_back({static_cast<size_t>(l) * region, bytes});
        s.push_back({static_cast<size_t>(nb + l) * region, bytes});
    }
    return s;
}

// A worker's two pinned staging buffers and their copy events.  The buffers are
// pinned once per process (portable, so any device's copies may use them) and
// kept: pinning 128 MB costs tens of milliseconds, a noticeable share of a
// 1 GB save.  Events belong to the calling device and live for one call.
struct Staging {
    void* buf[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    ~Staging() {
        for (int i = 0; i < 2; ++i)
            if (ev[i]) cudaEventDestroy(ev[i]);
    }
    bool init(int worker) {
        static void* pool[kWorkers][2] = {};
        for (int i = 0; i < 2; ++i) {
            if (!pool[worker][i] && cudaHostAlloc(&pool[worker][i], kChunk, cudaHostAllocPortable) != cudaSuccess) {
                pool[worker][i] = nullptr;
                cudaGetLastError();
                return false;
            }
            buf[i] = pool[worker][i];
            if (cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming) != cudaSuccess) {
                ev[i] = nullptr;
                cudaGetLastError();
                return false;
            }
        }
        return true;
    }
};

// Calls share the process's staging buffers, so they run one at a time.
std::mutex g_sess_mu;

// Chunks of the spans, each at most kChunk bytes, with their file offsets.
struct Piece {
    size_t off_bytes;   // byte offset in the blob
    size_t bytes;
    size_t file_off;    // byte offset in the file
};
std::vector<Piece> pieces_of(const std::vector<Span>& spans) {
    std::vector<Piece> p;
    size_t fo = kHeader;
    for (const Span& s : spans)
        for (size_t b = 0; b < s.bytes; b += kChunk) {
            const size_t n = std::min(kChunk, s.bytes - b);
            p.push_back({s.off * 2 + b, n, fo});
            fo += n;
        }
    return p;
}

bool write_full(int fd, const void* buf, size_t n, size_t off) {
    const char* c = static_cast<const char*>(buf);
    while (n > 0) {
        const ssize_t w = pwrite(fd, c, n, static_cast<off_t>(off));
        if (w <= 0) return false;
        c += w;
        n -= static_cast<size_t>(w);
        off += static_cast<size_t>(w);
    }
    return true;
}

bool read_full(int fd, void* buf, size_t n, size_t off) {
    char* c = static_cast<char*>(buf);
    while (n > 0) {
        const ssize_t r = pread(fd, c, n, static_cast<off_t>(off));
        if (r <= 0) return false;
        c += r;
        n -= static_cast<size_t>(r);
        off += static_cast<size_t>(r);
    }
    return true;
}

// Moves every kWorkers-th piece, starting at piece w, between the blob and the file.  save: device -> staging
// -> pwrite; load: pread -> staging -> device.  Each worker double-buffers: piece j's device copy overlaps the
// file I/O of the worker's previous piece.  Copies go on the caller's stream (issued from several threads they
// run in issue order, which only serialises the PCIe part).  First failure wins; the others stop at their next
// piece.
void worker(bool save, int w, int nw, int device, const std::vector<Piece>* pieces, char* blob, int fd,
            cudaStream_t st, Staging* sg, std::atomic<int>* failed, std::string* msg) {
    cudaSetDevice(device);   // a new thread starts on device 0; the caller's stream and blob may be elsewhere
    std::vector<size_t> mine;
    for (size_t i = static_cast<size_t>(w); i < pieces->size(); i += nw) mine.push_back(i);
    auto fail = [&](const std::string& m) {
        int z = 0;
        if (failed->compare_exchange_strong(z, 1)) *msg = m;
    };
    for (size_t k = 0; k <= mine.size() && !failed->load(); ++k) {
        if (save) {
            if (k < mine.size()) {
                const Piece& pc = (*pieces)[mine[k]];
                if (cudaMemcpyAsync(sg->buf[k % 2], blob + pc.off_bytes, pc.bytes, cudaMemcpyDeviceToHost, st) !=
                        cudaSuccess ||
                    cudaEventRecord(sg->ev[k % 2], st) != cudaSuccess) {
                    fail(std::string("device copy failed: ") + cudaGetErrorString(cudaGetLastError()));
                    break;
                }
            }
            if (k >= 1) {
                const Piece& pp = (*pieces)[mine[k - 1]];
                if (cudaEventSynchronize(sg->ev[(k - 1) % 2]) != cudaSuccess) {
                    fail(std::string("device copy failed: ") + cudaGetErrorString(cudaGetLastError()));
                    break;
                }
                if (!write_full(fd, sg->buf[(k - 1) % 2], pp.bytes, pp.file_off)) {
                    fail("file write failed");
                    break;
                }
            }
        } else if (k < mine.size()) {
            const Piece& pc = (*pieces)[mine[k]];
            // buffer k % 2 last fed piece k - 2's device copy
            if (k >= 2 && cudaEventSynchronize(sg->ev[k % 2]) != cudaSuccess) {
                fail(std::string("device copy failed: ") + cudaGetErrorString(cudaGetLastError()));
                break;
            }
            if (!read_full(fd, sg->buf[k % 2], pc.bytes, pc.file_off)) {
                fail("file is truncated");
                break;
            }
            if (cudaMemcpyAsync(blob + pc.off_bytes, sg->buf[k % 2], pc.bytes, cudaMemcpyHostToDevice, st) !=
                    cudaSuccess ||
                cudaEventRecord(sg->ev[k % 2], st) != cudaSuccess) {
                fail(std::string("device copy failed: ") + cudaGetErrorString(cudaGetLastError()));
                break;
            }
        }
    }
}

// Runs the workers; returns false with msg set on the first failure.  Every copy has finished on return, so the
// staging buffers are free for the next call.
bool move_pieces(bool save, const std::vector<Piece>& pieces, char* blob, int fd, cudaStream_t st,
                 std::string& msg) {
    if (pieces.empty()) return true;
    std::lock_guard<std::mutex> lock(g_sess_mu);
    // writes to one file serialise on its inode in the kernel, so a save uses one writer (its device copies
    // still run ahead of it); reads do not, so a load spreads over kWorkers readers
    const int nw = save ? 1 : static_cast<int>(std::min<size_t>(kWorkers, pieces.size()));
    std::vector<Staging> sg(nw);
    for (int w = 0; w < nw; ++w)
        if (!sg[w].init(w)) {
            msg = "pinned staging allocation failed";
            return false;
        }
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) {
        msg = "no current device";
        return false;
    }
    std::atomic<int> failed{0};
    std::vector<std::thread> th;
    for (int w = 0; w < nw; ++w)
        th.emplace_back(worker, save, w, nw, device, &pieces, blob, fd, st, &sg[w], &failed, &msg);
    for (std::thread& t : th) t.join();
    const cudaError_t e = cudaStreamSynchronize(st);
    if (!failed.load() && e != cudaSuccess) {
        msg = std::string("device copy failed: ") + cudaGetErrorString(e);
        return false;
    }
    return !failed.load();
}

bool check_geometry(uint32_t nb, uint32_t kv_dim, uint32_t max_seq, char* err, size_t errlen, const char* who) {
    if (nb == 0 || kv_dim == 0 || max_seq == 0) {
        set_err(err, errlen, "%s: bad geometry n_blocks=%u kv_dim=%u max_seq=%u", who, nb, kv_dim, max_seq);
        return false;
    }
    return true;
}

}  // namespace
}  // namespace yattn

using namespace yattn;

extern "C" int yattn_sess_kv_save(const uint16_t* kv_dev, uint32_t n_blocks, uint32_t kv_dim, uint32_t max_seq,
                                  uint32_t pos, const char* path, void* stream, char* err, size_t errlen) {
    const char* who = "sess_kv_save";
    if (!kv_dev || !path) {
        set_err(err, errlen, "%s: null argument", who);
        return -1;
    }
    if (!check_geometry(n_blocks, kv_dim, max_seq, err, errlen, who)) return -1;
    if (pos > max_seq) {
        set_err(err, errlen, "%s: pos %u > max_seq %u", who, pos, max_seq);
        return -1;
    }
    const int fd = open(path, O_WRONLY | O_CREAT | O_TRUNC, 0644);
    if (fd < 0) {
        set_err(err, errlen, "%s: cannot open %s", who, path);
        return -1;
    }
    char head[kHeader];
    const uint32_t hdr[4] = {n_blocks, kv_dim, max_seq, pos};
    memcpy(head, kMagic, 8);
    memcpy(head + 8, hdr, 16);
    std::string msg;
    bool ok = write_full(fd, head, kHeader, 0);
    if (!ok) msg = "file write failed";
    if (ok)
        ok = move_pieces(true, pieces_of(spans_of(n_blocks, kv_dim, max_seq, pos)),
                         const_cast<char*>(reinterpret_cast<const char*>(kv_dev)), fd, static_cast<cudaStream_t>(stream),
                         msg);
    if (close(fd) != 0 && ok) {
        ok = false;
        msg = "closing the file failed";
    }
    if (ok) return 0;
    set_err(err, errlen, "%s: %s: %s", who, path, msg.c_str());
    return -1;
}

extern "C" int yattn_sess_kv_load(uint16_t* kv_dev, uint32_t n_blocks, uint32_t kv_dim, uint32_t max_seq,
                                  const char* path, uint32_t* pos, void* stream, char* err, size_t errlen) {
    const char* who = "sess_kv_load";
    if (!kv_dev || !path) {
        set_err(err, errlen, "%s: null argument", who);
        return -1;
    }
    if (!check_geometry(n_blocks, kv_dim, max_seq, err, errlen, who)) return -1;
    const int fd = open(path, O_RDONLY);
    if (fd < 0) {
        set_err(err, errlen, "%s: cannot open %s", who, path);
        return -1;
    }
    char head[kHeader];
    uint32_t hdr[4];
    if (!read_full(fd, head, kHeader, 0) || memcmp(head, kMagic, 8) != 0) {
        close(fd);
        set_err(err, errlen, "%s: %s is not a session KV file", who, path);
        return -1;
    }
    memcpy(hdr, head + 8, 16);
    // the reference refuses a file made by another model or configuration (cache.c:229-233)
    if (hdr[0] != n_blocks || hdr[1] != kv_dim || hdr[2] != max_seq || hdr[3] > max_seq) {
        close(fd);
        set_err(err, errlen, "%s: file has n_blocks=%u kv_dim=%u max_seq=%u pos=%u, engine n_blocks=%u kv_dim=%u "
                "max_seq=%u", who, hdr[0], hdr[1], hdr[2], hdr[3], n_blocks, kv_dim, max_seq);
        return -1;
    }
    std::string msg;
    const bool ok = move_pieces(false, pieces_of(spans_of(n_blocks, kv_dim, max_seq, hdr[3])),
                                reinterpret_cast<char*>(kv_dev), fd, static_cast<cudaStream_t>(stream), msg);
    close(fd);
    if (!ok) {
        set_err(err, errlen, "%s: %s: %s", who, path, msg.c_str());
        return -1;
    }
    if (pos) *pos = hdr[3];
    return 0;
}
