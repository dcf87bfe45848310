// Packed layer files: a layer's weights on disk in the exact byte layout the kernels stream.
//
// The reference caches dequantized device tensors on disk (native/glm53/deq_cache.vyb:1-93:
// one .bin of raw f64 bytes per tensor, re-uploaded on later runs), because its trellis
// dequantization dominated load time.  Here nothing is dequantized at load at all: the file
// holds the router and the expert stacks as the kernels read them (stage-tiled Q8_0 from
// vfmoe_q8_0_tile, or the EXL3 trellis + suh/svh as stored), so a load is one sequential read
// into device memory and the descriptor points into it.
//
// File layout (little-endian):
//   header, 4096 bytes: "VFMOEPK1", u32 version, u32 section count, then the layer descriptor
//   words (vfmoe_layer_desc with every device pointer replaced by a byte offset into the data
//   region; 0 for a matrix that is absent, since only router_w starts at offset 0), then per
//   section {u64 offset, u64 bytes}.
//   data region from byte 4096: sections, each 4096-aligned: router_w, router_bias, then for
//   each of gate, up, down, sh_gate, sh_up, sh_down: data, suh, svh (EXL3) as present.
// A section's bytes are the full stack (n_local experts x expert_stride, or one matrix).
#include <cstdio>
#include <cstring>
#include <vector>

#include "common.cuh"

namespace vfmoe {

static const char kMagic[8] = {'V', 'F', 'M', 'O', 'E', 'P', 'K', '1'};
constexpr uint32_t kPackVersion = 1;
constexpr int64_t kPackAlign = 4096;
constexpr int kMaxSections = 2 + 6 * 3;

struct PackSection {
    int64_t *desc_word;  // the descriptor word that holds this section's pointer
    int64_t bytes;
};

// Every device range a descriptor references, with its byte size.
static int desc_sections(vfmoe_layer_desc &d, std::vector<PackSection> &out) {
    out.clear();
    const int64_t H = d.hidden, I = d.inter, E = d.n_local_experts ? d.n_local_experts : d.n_experts;
    out.push_back({&d.router_w, d.n_experts * H * 4});
    out.push_back({&d.router_bias, d.n_experts * 4});
    vfmoe_matrix *ms[6] = {&d.gate, &d.up, &d.down, &d.sh_gate, &d.sh_up, &d.sh_down};
    const int64_t kk[3] = {H, H, I}, nn[3] = {I, I, H};
    for (int i = 0; i < 6; ++i) {
        vfmoe_matrix &m = *ms[i];
        if (!m.data) continue;
        const int64_t K = kk[i % 3], N = nn[i % 3];
        const int64_t count = i < 3 ? E : 1;
        const bool dense = i >= 3 && d.shared_format == VFMOE_WFMT_BF16;
        int64_t one;
        if (dense)
            one = N * K * 2;  // bf16 rows [out][in]
        else if (d.weight_format == VFMOE_WFMT_EXL3)
            one = K / 16 * (N / 16) * 2 * 16 * d.exl3_bits;
        else
            one = N * (K / 32 * 34);  // Q8_0 rows = output channels
        const int64_t stride = count > 1 ? m.expert_stride : one;
        if (stride < one) {
            set_error("packed layer: matrix %d stride %lld < %lld bytes", i, (long long)stride, (long long)one);
            return VFMOE_ERR_INVALID;
        }
        out.push_back({&m.data, count > 1 ? stride * (count - 1) + one : one});
        if (d.weight_format == VFMOE_WFMT_EXL3 && !dense) {
            const int64_t ss = count > 1 ? m.suh_stride : K * 2, vs = count > 1 ? m.svh_stride : N * 2;
            out.push_back({&m.suh, count > 1 ? ss * (count - 1) + K * 2 : K * 2});
            out.push_back({&m.svh, count > 1 ? vs * (count - 1) + N * 2 : N * 2});
        }
    }
    return VFMOE_OK;
}

struct PackHeader {
    char magic[8];
    uint32_t version, n_sections;
    vfmoe_layer_desc desc;  // pointers as byte offsets into the data region
    int64_t sec_off[kMaxSections];
    int64_t sec_bytes[kMaxSections];
};
static_assert(sizeof(PackHeader) <= kPackAlign, "header fits its block");

static int read_header(FILE *f, PackHeader &h, const char *path) {
    char block[kPackAlign];
    if (fread(block, 1, kPackAlign, f) != (size_t)kPackAlign) {
        set_error("packed layer %s: short header", path);
        return VFMOE_ERR_INVALID;
    }
    memcpy(&h, block, sizeof(h));
    if (memcmp(h.magic, kMagic, 8) || h.version != kPackVersion || h.n_sections > (uint32_t)kMaxSections) {
        set_error("packed layer %s: not a version-%u vfmoe pack", path, kPackVersion);
        return VFMOE_ERR_INVALID;
    }
    return VFMOE_OK;
}

// n bytes of f at offset off into dst: host memory by one read, or device memory through two
// pinned 32 MiB staging buffers, each chunk's copy overlapping the next chunk's read.
// Synchronous.  `what` names the source in error messages.
int read_range(FILE *f, int64_t off, int64_t n, char *dst, bool device, const char *what) {
    if (fseek(f, off, SEEK_SET) != 0) {
        set_error("%s: seek to %lld failed", what, (long long)off);
        return VFMOE_ERR_INVALID;
    }
    if (!device) {
        if (n > 0 && fread(dst, 1, n, f) != (size_t)n) {
            set_error("%s: short read", what);
            return VFMOE_ERR_INVALID;
        }
        return VFMOE_OK;
    }
    if (n == 0) return VFMOE_OK;
    const int64_t chunk = 32 << 20;
    char *stage = nullptr;
    cudaEvent_t done[2] = {nullptr, nullptr};
    cudaStream_t st = nullptr;
    int rc = VFMOE_OK;
    cudaError_t e = cudaHostAlloc(&stage, 2 * std::min<int64_t>(chunk, n), cudaHostAllocDefault);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done[0], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&done[1], cudaEventDisableTiming);
    if (e != cudaSuccess) rc = cuda_fail(e, "staging for a device read", __FILE__, __LINE__);
    const int64_t cs = std::min<int64_t>(chunk, n);
    bool used[2] = {false, false};
    int which = 0;
    for (int64_t p = 0; !rc && p < n; p += cs) {
        const int64_t m = std::min(cs, n - p);
        char *buf = stage + which * cs;
        if (used[which] && (e = cudaEventSynchronize(done[which])) != cudaSuccess) {
            rc = cuda_fail(e, "device read", __FILE__, __LINE__);
            break;
        }
        if (fread(buf, 1, m, f) != (size_t)m) {
            set_error("%s: short read", what);
            rc = VFMOE_ERR_INVALID;
            break;
        }
        e = cudaMemcpyAsync(dst + p, buf, m, cudaMemcpyHostToDevice, st);
        if (e == cudaSuccess) e = cudaEventRecord(done[which], st);
        if (e != cudaSuccess) {
            rc = cuda_fail(e, "device read", __FILE__, __LINE__);
            break;
        }
        used[which] = true;
        which ^= 1;
    }
    if (st) {
        e = cudaStreamSynchronize(st);
        if (!rc && e != cudaSuccess) rc = cuda_fail(e, "device read", __FILE__, __LINE__);
        cudaStreamDestroy(st);
    }
    for (int b = 0; b < 2; ++b)
        if (done[b]) cudaEventDestroy(done[b]);
    if (stage) cudaFreeHost(stage);
    return rc;
}

}  // namespace vfmoe

using namespace vfmoe;

extern "C" {

int vfmoe_pack_save(const char *path, const vfmoe_layer_desc *desc) {
    if (!path || !desc) {
        set_error("vfmoe_pack_save: bad arguments");
        return VFMOE_ERR_INVALID;
    }
    PackHeader h{};
    memcpy(h.magic, kMagic, 8);
    h.version = kPackVersion;
    h.desc = *desc;
    std::vector<PackSection> secs;
    if (int rc = desc_sections(h.desc, secs)) return rc;
    h.n_sections = (uint32_t)secs.size();
    std::vector<int64_t> src(secs.size());
    int64_t off = 0;
    for (size_t i = 0; i < secs.size(); ++i) {
        src[i] = *secs[i].desc_word;
        h.sec_off[i] = off;
        h.sec_bytes[i] = secs[i].bytes;
        *secs[i].desc_word = off;  // the file stores offsets
        off = align_up(off + secs[i].bytes, kPackAlign);
    }
    FILE *f = fopen(path, "wb");
    if (!f) {
        set_error("vfmoe_pack_save: cannot open %s for writing", path);
        return VFMOE_ERR_INVALID;
    }
    std::vector<char> block(kPackAlign, 0);
    memcpy(block.data(), &h, sizeof(h));
    bool ok = fwrite(block.data(), 1, kPackAlign, f) == (size_t)kPackAlign;
    const int64_t chunk = 64 << 20;
    std::vector<char> buf(chunk);
    const std::vector<char> zeros(kPackAlign, 0);
    int rc = VFMOE_OK;
    for (size_t i = 0; i < secs.size() && ok; ++i) {
        for (int64_t p = 0; p < secs[i].bytes && ok; p += chunk) {
            const int64_t n = std::min(chunk, secs[i].bytes - p);
            cudaError_t e = cudaMemcpy(buf.data(), reinterpret_cast<const char *>(src[i]) + p, n, cudaMemcpyDeviceToHost);
            if (e != cudaSuccess) {
                rc = cuda_fail(e, "vfmoe_pack_save: device read", __FILE__, __LINE__);
                ok = false;
                break;
            }
            ok = fwrite(buf.data(), 1, n, f) == (size_t)n;
        }
        const int64_t pad = align_up(secs[i].bytes, kPackAlign) - secs[i].bytes;
        if (ok && pad) ok = fwrite(zeros.data(), 1, pad, f) == (size_t)pad;
    }
    if (fclose(f) != 0) ok = false;
    if (rc) return rc;
    if (!ok) {
        set_error("vfmoe_pack_save: write to %s failed", path);
        return VFMOE_ERR_INVALID;
    }
    return VFMOE_OK;
}

int64_t vfmoe_pack_bytes(const char *path) {
    FILE *f = path ? fopen(path, "rb") : nullptr;
    if (!f) {
        set_error("vfmoe_pack_bytes: cannot open %s", path ? path : "(null)");
        return VFMOE_ERR_INVALID;
    }
    PackHeader h;
    const int rc = read_header(f, h, path);
    fclose(f);
    if (rc) return rc;
    int64_t end = 0;
    for (uint32_t i = 0; i < h.n_sections; ++i) end = std::max(end, h.sec_off[i] + h.sec_bytes[i]);
    return align_up(end, 256);
}

int vfmoe_pack_load(const char *path, int64_t dev_base, int64_t dev_bytes, vfmoe_layer_desc *desc_out) {
    if (!path || !dev_base || (dev_base & 255) || !desc_out) {
        set_error("vfmoe_pack_load: bad arguments (256-byte aligned device buffer required)");
        return VFMOE_ERR_INVALID;
    }
    FILE *f = fopen(path, "rb");
    if (!f) {
        set_error("vfmoe_pack_load: cannot open %s", path);
        return VFMOE_ERR_INVALID;
    }
    PackHeader h;
    int rc = read_header(f, h, path);
    vfmoe_layer_desc d = h.desc;
    std::vector<PackSection> secs;
    if (!rc) rc = desc_sections(d, secs);
    if (!rc && secs.size() != h.n_sections) {
        set_error("vfmoe_pack_load: %s: section table does not match its descriptor", path);
        rc = VFMOE_ERR_INVALID;
    }
    int64_t need = 0;
    for (uint32_t i = 0; !rc && i < h.n_sections; ++i) {
        if (*secs[i].desc_word != h.sec_off[i] || secs[i].bytes != h.sec_bytes[i] || h.sec_off[i] % kPackAlign) {
            set_error("vfmoe_pack_load: %s: section %u inconsistent", path, i);
            rc = VFMOE_ERR_INVALID;
        }
        need = std::max(need, h.sec_off[i] + h.sec_bytes[i]);
    }
    if (!rc && need > dev_bytes) {
        set_error("vfmoe_pack_load: %s needs %lld device bytes, buffer has %lld", path, (long long)need,
                  (long long)dev_bytes);
        rc = VFMOE_ERR_WORKSPACE;
    }
    for (uint32_t i = 0; !rc && i < h.n_sections; ++i)
        rc = read_range(f, kPackAlign + h.sec_off[i], h.sec_bytes[i], reinterpret_cast<char *>(dev_base) + h.sec_off[i],
                        true, path);
    fclose(f);
    if (rc) return rc;
    for (auto &s : secs) *s.desc_word = dev_base + *s.desc_word;
    *desc_out = d;
    return VFMOE_OK;
}

}  // extern "C"
