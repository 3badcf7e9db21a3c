// The snn_b200 CSR file: a network saved once (by the reference's builders,
// snn_b200_network_wrap views, or a downloaded device topology) and mapped
// read-only afterwards, so large networks are not rebuilt for every run and
// STREAMING contexts copy their rows straight from the page cache (the
// library page-locks the mapping read-only when the OS allows it).
//
// Layout (little-endian, native widths), every section 4096-byte aligned:
//   [0, 4096)        header (CsrFileHeader, zero padded)
//   row_ptr_offset   u64 row_ptr[n + 1]
//   col_idx_offset   u64 col_idx[e]
//   weights_offset   f32 weights[e]
// A mapped network is validated like snn_build_custom_csr (src/snn.c:158-180)
// before it is returned, so a damaged file cannot reach a kernel.
#include "b200_network.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <unordered_map>

namespace {

constexpr char kMagic[8] = {'S', 'N', 'N', 'C', 'S', 'R', '0', '1'};
constexpr uint32_t kVersion = 1;
constexpr uint64_t kAlign = 4096;

struct CsrFileHeader {
    char magic[8];
    uint32_t version;
    uint32_t header_bytes;
    uint64_t neuron_count;
    uint64_t synapse_count;
    int32_t architecture;
    snn_lif_params_t lif;
    float decay;
    uint64_t row_ptr_offset;
    uint64_t col_idx_offset;
    uint64_t weights_offset;
    uint64_t file_bytes;
};
static_assert(sizeof(CsrFileHeader) <= kAlign, "header fits its block");

uint64_t align_up(uint64_t x) { return (x + kAlign - 1) / kAlign * kAlign; }

struct Mapping {
    void *base;
    size_t bytes;
};
std::mutex g_map_mu;
std::unordered_map<const snn_network_t *, Mapping> g_maps;

bool write_all(int fd, const void *data, uint64_t bytes) {
    const char *p = static_cast<const char *>(data);
    while (bytes) {
        const size_t chunk = bytes > (1ull << 30) ? (1ull << 30) : (size_t)bytes;
        const ssize_t w = ::write(fd, p, chunk);
        if (w < 0) {
            if (errno == EINTR) continue;
            return false;
        }
        p += w;
        bytes -= (uint64_t)w;
    }
    return true;
}

bool pad_to(int fd, uint64_t *pos, uint64_t target) {
    static const char zeros[kAlign] = {};
    while (*pos < target) {
        const uint64_t k = target - *pos < kAlign ? target - *pos : kAlign;
        if (!write_all(fd, zeros, k)) return false;
        *pos += k;
    }
    return true;
}

}  // namespace

namespace b200host {

bool lif_valid(const snn_lif_params_t *p) {
    return p && std::isfinite(p->dt_ms) && std::isfinite(p->membrane_tau_ms) && std::isfinite(p->v_rest) &&
           std::isfinite(p->v_reset) && std::isfinite(p->v_threshold) && std::isfinite(p->input_scale) &&
           p->dt_ms > 0.0f && p->membrane_tau_ms > 0.0f && p->v_threshold > p->v_reset;
}

snn_status_t validate_csr(uint64_t n, uint64_t e, const uint64_t *row_ptr, const uint64_t *col, const float *w) {
    if (n == 0 || row_ptr == nullptr || (e != 0 && (col == nullptr || w == nullptr))) return SNN_ERR_INVALID_ARGUMENT;
    if (row_ptr[0] != 0 || row_ptr[n] != e) return SNN_ERR_INVALID_ARGUMENT;
    for (uint64_t i = 0; i < n; ++i)
        if (row_ptr[i] > row_ptr[i + 1] || row_ptr[i + 1] > e) return SNN_ERR_INVALID_ARGUMENT;
    for (uint64_t i = 0; i < e; ++i)
        if (col[i] >= n || !std::isfinite(w[i])) return SNN_ERR_INVALID_ARGUMENT;
    return SNN_OK;
}

bool release_mapping(snn_network_t *network) {
    Mapping m{};
    {
        std::lock_guard<std::mutex> lock(g_map_mu);
        auto it = g_maps.find(network);
        if (it == g_maps.end()) return false;
        m = it->second;
        g_maps.erase(it);
    }
    munmap(m.base, m.bytes);
    delete network;
    return true;
}

}  // namespace b200host

extern "C" {

snn_status_t snn_b200_network_save(const snn_network_t *net, const char *path) {
    if (net == nullptr || path == nullptr || net->neuron_count == 0 || net->row_ptr == nullptr ||
        (net->synapse_count && (net->col_idx == nullptr || net->weights == nullptr)))
        return SNN_ERR_INVALID_ARGUMENT;
    const uint64_t n = net->neuron_count, e = net->synapse_count;
    if (n > (UINT64_MAX - kAlign) / 8 - 1 || e > (UINT64_MAX / 4 - 4 * kAlign) / 3) return SNN_ERR_OVERFLOW;
    CsrFileHeader h{};
    std::memcpy(h.magic, kMagic, sizeof(kMagic));
    h.version = kVersion;
    h.header_bytes = (uint32_t)kAlign;
    h.neuron_count = n;
    h.synapse_count = e;
    h.architecture = (int32_t)net->architecture;
    h.lif = net->lif;
    h.decay = net->decay;
    h.row_ptr_offset = kAlign;
    h.col_idx_offset = align_up(h.row_ptr_offset + (n + 1) * 8);
    h.weights_offset = align_up(h.col_idx_offset + e * 8);
    h.file_bytes = h.weights_offset + e * 4;
    // Written to a temporary name and renamed, so a reader never maps a
    // partly written file under the final name.
    const std::string tmp = std::string(path) + ".partial";
    const int fd = ::open(tmp.c_str(), O_WRONLY | O_CREAT | O_TRUNC, 0644);
    if (fd < 0) return SNN_ERR_INVALID_ARGUMENT;
    uint64_t pos = sizeof(h);
    bool ok = write_all(fd, &h, sizeof(h));
    ok = ok && pad_to(fd, &pos, h.row_ptr_offset) && write_all(fd, net->row_ptr, (n + 1) * 8);
    pos = h.row_ptr_offset + (n + 1) * 8;
    ok = ok && pad_to(fd, &pos, h.col_idx_offset) && write_all(fd, net->col_idx, e * 8);
    pos = h.col_idx_offset + e * 8;
    ok = ok && pad_to(fd, &pos, h.weights_offset) && write_all(fd, net->weights, e * 4);
    ok = (::close(fd) == 0) && ok;
    if (!ok || std::rename(tmp.c_str(), path) != 0) {
        ::unlink(tmp.c_str());
        return SNN_ERR_OUT_OF_MEMORY;
    }
    return SNN_OK;
}

snn_status_t snn_b200_network_map(const char *path, snn_network_t **out) {
    if (out == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    *out = nullptr;
    if (path == nullptr) return SNN_ERR_INVALID_ARGUMENT;
    const int fd = ::open(path, O_RDONLY);
    if (fd < 0) return SNN_ERR_INVALID_ARGUMENT;
    struct stat sb {};
    if (fstat(fd, &sb) != 0 || (uint64_t)sb.st_size < kAlign) {
        ::close(fd);
        return SNN_ERR_INVALID_ARGUMENT;
    }
    const size_t bytes = (size_t)sb.st_size;
    void *base = mmap(nullptr, bytes, PROT_READ, MAP_SHARED, fd, 0);
    ::close(fd);  // the mapping keeps the file open
    if (base == MAP_FAILED) return SNN_ERR_OUT_OF_MEMORY;
    auto fail = [&](snn_status_t st) {
        munmap(base, bytes);
        return st;
    };
    CsrFileHeader h{};
    std::memcpy(&h, base, sizeof(h));
    const uint64_t n = h.neuron_count, e = h.synapse_count;
    if (std::memcmp(h.magic, kMagic, sizeof(kMagic)) != 0 || h.version != kVersion || h.header_bytes != kAlign ||
        n == 0 || n > (UINT64_MAX - kAlign) / 8 - 1 || e > (UINT64_MAX / 4 - 4 * kAlign) / 3 ||
        h.row_ptr_offset != kAlign || h.col_idx_offset != align_up(h.row_ptr_offset + (n + 1) * 8) ||
        h.weights_offset != align_up(h.col_idx_offset + e * 8) || h.file_bytes != h.weights_offset + e * 4 ||
        h.file_bytes > bytes || !b200host::lif_valid(&h.lif) || !std::isfinite(h.decay))
        return fail(SNN_ERR_INVALID_ARGUMENT);
    char *b = static_cast<char *>(base);
    const uint64_t *row_ptr = reinterpret_cast<const uint64_t *>(b + h.row_ptr_offset);
    const uint64_t *col = reinterpret_cast<const uint64_t *>(b + h.col_idx_offset);
    const float *w = reinterpret_cast<const float *>(b + h.weights_offset);
    madvise(base, bytes, MADV_SEQUENTIAL);
    const snn_status_t st = b200host::validate_csr(n, e, row_ptr, e ? col : nullptr, e ? w : nullptr);
    if (st != SNN_OK) return fail(st);
    madvise(base, bytes, MADV_NORMAL);
    snn_network_t *net = new (std::nothrow) snn_network_t();
    if (net == nullptr) return fail(SNN_ERR_OUT_OF_MEMORY);
    net->neuron_count = n;
    net->synapse_count = e;
    net->architecture = (snn_architecture_t)h.architecture;
    net->lif = h.lif;
    net->decay = h.decay;  // as saved: the network's own decay (src/snn.c:111-113)
    net->row_ptr = const_cast<uint64_t *>(row_ptr);
    net->col_idx = const_cast<uint64_t *>(col);
    net->weights = const_cast<float *>(w);
    {
        std::lock_guard<std::mutex> lock(g_map_mu);
        g_maps[net] = Mapping{base, bytes};
    }
    *out = net;
    return SNN_OK;
}

}  // extern "C"
