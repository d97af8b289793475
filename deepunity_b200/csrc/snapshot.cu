// snapshot.cu -- KV-cache snapshots (device <-> file) and the native loader of an
// import_params.py export folder.
//
// * du_model_load_folder replaces MiniCPM5Weights' upload pump
//   (InferenceEngine/LLM/MiniCPM5/MiniCPM5Weights.cs:315-380): every "*.bin"
//   under the folder is memory-mapped and placed by its relative name, exactly
//   as du_model_load_tensor places it.
// * du_model_save_cache / du_model_load_cache keep MiniCPM5Cache's "M5KV"
//   version-1 folder (MiniCPM5Cache.cs:31-32, 78-200): meta.bin = int32 magic
//   0x4D354B56, version 1, layers, kv heads, head_dim, tokens; then
//   k_cache_layer_<i>.bin / v_cache_layer_<i>.bin, tokens x kv heads x head_dim
//   fp16 values, position-major.  The fp16 cache is written as stored; loading
//   follows the reference reader (HalfBitsToFloat): fp16 subnormals become
//   signed zero.  Every file is validated before anything is uploaded, and a
//   mismatch is a miss, not an error.  The reference persists only an fp32
//   cache in this format; the INT8 cache is not written to it (a miss on load).
// * du_model_save_kv / du_model_load_kv / du_kv_file_peek: one file per
//   sequence, the layout of the reference's version-2 prompt cache
//   (Qwen3_5Cache.cs:149-170) for a model whose layers are all full attention:
//     uint32 magic 'LMKV'  int32 version 2  uint64 context hash  uint8 kv format
//     int32 tokens  int32 layers  int32 extra length + extra bytes
//     per layer: uint8 kind (0), then length-prefixed blobs: K rows, V rows
//     (tokens x row bytes), and with the INT8 cache the K and V scale /
//     zero-point words (tokens x kv heads x 4 bytes).
//   It is written to <path>.tmp and renamed over <path>, so a torn write never
//   shadows a good snapshot.  The hash is the caller's identity of the cached
//   context (weights, cache format, prompt); any mismatch is a miss.
#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "model_state.h"

namespace du {

int place_tensor(du_model *m, const char *name, const void *src, size_t bytes, cudaMemcpyKind kind);

static constexpr int32_t M5KV_MAGIC = 0x4D354B56;     // "M5KV"
static constexpr int32_t M5KV_VERSION = 1;
static constexpr uint32_t LMKV_MAGIC = 0x4C4D4B56;    // "LMKV"
static constexpr int32_t LMKV_VERSION = 2;

// ------------------------------------------------------------------ helpers

static int mkdirs(const std::string &dir)
{
    std::string cur;
    for (size_t i = 0; i <= dir.size(); i++) {
        if (i == dir.size() || dir[i] == '/') {
            if (!cur.empty() && mkdir(cur.c_str(), 0755) != 0 && errno != EEXIST)
                return fail(DU_EIO, "cannot create directory " + cur + ": " + strerror(errno));
        }
        if (i < dir.size()) cur += dir[i];
    }
    return DU_OK;
}

static bool read_file(const std::string &path, std::vector<uint8_t> &out, size_t expect = (size_t)-1)
{
    FILE *f = fopen(path.c_str(), "rb");
    if (!f) return false;
    fseek(f, 0, SEEK_END);
    const long n = ftell(f);
    fseek(f, 0, SEEK_SET);
    bool ok = n >= 0 && (expect == (size_t)-1 || (size_t)n == expect);
    if (ok) {
        out.resize((size_t)n);
        ok = n == 0 || fread(out.data(), 1, (size_t)n, f) == (size_t)n;
    }
    fclose(f);
    return ok;
}

static int write_file(const std::string &path, const void *data, size_t n)
{
    const std::string tmp = path + ".tmp";
    FILE *f = fopen(tmp.c_str(), "wb");
    if (!f) return fail(DU_EIO, "cannot write " + tmp + ": " + strerror(errno));
    const bool ok = n == 0 || fwrite(data, 1, n, f) == n;
    if (fclose(f) != 0 || !ok) {
        unlink(tmp.c_str());
        return fail(DU_EIO, "write failed: " + tmp);
    }
    if (rename(tmp.c_str(), path.c_str()) != 0) {
        unlink(tmp.c_str());
        return fail(DU_EIO, "cannot rename " + tmp + ": " + strerror(errno));
    }
    return DU_OK;
}

// HalfBitsToFloat of the reference reader (MiniCPM5Cache.cs:239-246): subnormals -> signed zero
static void flush_fp16_subnormals(uint16_t *h, size_t n)
{
    for (size_t i = 0; i < n; i++)
        if ((h[i] & 0x7C00u) == 0) h[i] &= 0x8000u;
}

// bytes of one sequence's cache rows of one layer, and where they start
struct SeqKv {
    size_t row_bytes;          // one position's K (or V) row: hkv_l x hd elements
    size_t sz_bytes;           // one position's scale / zero-point words (INT8 cache)
    uint8_t *k, *v;            // layer l, position 0 of the sequence
    uint8_t *ksz, *vsz;
};

static SeqKv seq_kv(du_model *m, int seq, int l)
{
    SeqKv s = {};
    const size_t pos0 = (size_t)seq * m->cap * m->hkv_l;      // first (position, kv head) row of the sequence
    if (m->kv8) {
        const size_t rows = m->kv_layer_elems / m->hd;
        s.row_bytes = (size_t)m->hkv_l * m->hd;
        s.sz_bytes = (size_t)m->hkv_l * 4;
        s.k = m->k8 + (size_t)l * m->kv_layer_elems + pos0 * m->hd;
        s.v = m->v8 + (size_t)l * m->kv_layer_elems + pos0 * m->hd;
        s.ksz = reinterpret_cast<uint8_t *>(m->ksz + (size_t)l * rows + pos0);
        s.vsz = reinterpret_cast<uint8_t *>(m->vsz + (size_t)l * rows + pos0);
    } else {
        s.row_bytes = (size_t)m->hkv_l * m->hd * 2;
        s.k = reinterpret_cast<uint8_t *>(m->k_cache + (size_t)l * m->kv_layer_elems + pos0 * m->hd);
        s.v = reinterpret_cast<uint8_t *>(m->v_cache + (size_t)l * m->kv_layer_elems + pos0 * m->hd);
    }
    return s;
}

static int d2h(du_model *m, std::vector<uint8_t> &out, const void *src, size_t n)
{
    out.resize(n);
    if (n) DU_CUDA_TRY(cudaMemcpyAsync(out.data(), src, n, cudaMemcpyDeviceToHost, m->stream));
    return DU_OK;
}

// ------------------------------------------------------------ export folder

static void list_bins(const std::string &root, const std::string &rel, std::vector<std::string> &out, int depth)
{
    if (depth > 8) return;
    DIR *d = opendir((root + (rel.empty() ? "" : "/" + rel)).c_str());
    if (!d) return;
    std::vector<std::string> names;
    while (dirent *e = readdir(d)) {
        const std::string n = e->d_name;
        if (n == "." || n == "..") continue;
        names.push_back(n);
    }
    closedir(d);
    std::sort(names.begin(), names.end());
    for (const auto &n : names) {
        const std::string r = rel.empty() ? n : rel + "/" + n;
        struct stat st;
        if (stat((root + "/" + r).c_str(), &st) != 0) continue;
        if (S_ISDIR(st.st_mode)) list_bins(root, r, out, depth + 1);
        else if (S_ISREG(st.st_mode) && n.size() > 4 && n.compare(n.size() - 4, 4, ".bin") == 0) out.push_back(r);
    }
}

}  // namespace du

using namespace du;

extern "C" {

DU_API int du_model_load_folder(du_model *m, const char *folder, int *n_files)
{
    DU_GUARD(m);
    DU_CHECK_ARG(folder, "du_model_load_folder: null folder");
    if (n_files) *n_files = 0;
    std::vector<std::string> files;
    list_bins(folder, "", files, 0);
    if (files.empty()) return fail(DU_ENOTFOUND, std::string("no .bin tensors under ") + folder);
    int loaded = 0;
    for (const auto &rel : files) {
        const std::string path = std::string(folder) + "/" + rel;
        const int fd = open(path.c_str(), O_RDONLY);
        if (fd < 0) return fail(DU_EIO, "cannot open " + path);
        struct stat st;
        if (fstat(fd, &st) != 0 || st.st_size <= 0) {
            close(fd);
            return fail(DU_EIO, "cannot size (or empty) " + path);
        }
        void *p = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
        close(fd);
        if (p == MAP_FAILED) return fail(DU_EIO, "cannot map " + path);
        int rc = place_tensor(m, rel.c_str(), p, (size_t)st.st_size, cudaMemcpyHostToDevice);
        // the copies read the mapping until the stream has drained them
        const cudaError_t e = cudaStreamSynchronize(m->stream);
        munmap(p, (size_t)st.st_size);
        if (rc) return rc;
        if (e != cudaSuccess) return cuda_fail(e, "du_model_load_folder");
        loaded++;
    }
    if (n_files) *n_files = loaded;
    return DU_OK;
}

DU_API int du_model_save_cache(du_model *m, int seq, const char *folder)
{
    DU_GUARD(m);
    DU_CHECK_ARG(folder && seq >= 0 && seq < m->maxb, "du_model_save_cache: bad arguments");
    if (m->kv8) return fail(DU_ESTATE, "du_model_save_cache: the M5KV format holds fp16 rows; use du_model_save_kv");
    const int tokens = m->h_cache_len[seq];
    if (tokens <= 0) return DU_OK;                    // nothing cached: nothing written (as the reference)
    int rc = mkdirs(folder);
    if (rc) return rc;
    DU_CUDA_TRY(cudaStreamSynchronize(m->stream));
    std::vector<uint8_t> buf;
    for (int l = 0; l < m->L; l++) {
        const SeqKv s = seq_kv(m, seq, l);
        for (int kv = 0; kv < 2; kv++) {
            if ((rc = d2h(m, buf, kv ? s.v : s.k, (size_t)tokens * s.row_bytes))) return rc;
            DU_CUDA_TRY(cudaStreamSynchronize(m->stream));
            char name[64];
            snprintf(name, sizeof name, "/%s_cache_layer_%d.bin", kv ? "v" : "k", l);
            if ((rc = write_file(std::string(folder) + name, buf.data(), buf.size()))) return rc;
        }
    }
    // meta.bin last: a folder whose save was cut short has no header and loads as a miss
    const int32_t meta[6] = {M5KV_MAGIC, M5KV_VERSION, m->L, m->hkv_l, m->hd, tokens};
    return write_file(std::string(folder) + "/meta.bin", meta, sizeof meta);
}

DU_API int du_model_load_cache(du_model *m, int seq, const char *folder, int *loaded)
{
    DU_GUARD(m);
    DU_CHECK_ARG(folder && loaded && seq >= 0 && seq < m->maxb, "du_model_load_cache: bad arguments");
    *loaded = 0;
    if (m->kv8) return DU_OK;                         // not kept in this format: a miss
    std::vector<uint8_t> meta;
    if (!read_file(std::string(folder) + "/meta.bin", meta) || meta.size() < 24) return DU_OK;
    int32_t h[6];
    memcpy(h, meta.data(), sizeof h);
    if (h[0] != M5KV_MAGIC || h[1] != M5KV_VERSION || h[2] != m->L || h[3] != m->hkv_l || h[4] != m->hd) return DU_OK;
    const int tokens = h[5];
    if (tokens <= 0 || tokens > m->cap) return DU_OK;
    const size_t bytes = (size_t)tokens * m->hkv_l * m->hd * 2;
    // read and check every file before anything reaches the device
    std::vector<std::vector<uint8_t>> data((size_t)2 * m->L);
    for (int l = 0; l < m->L; l++)
        for (int kv = 0; kv < 2; kv++) {
            char name[64];
            snprintf(name, sizeof name, "/%s_cache_layer_%d.bin", kv ? "v" : "k", l);
            if (!read_file(std::string(folder) + name, data[(size_t)2 * l + kv], bytes)) return DU_OK;
            flush_fp16_subnormals(reinterpret_cast<uint16_t *>(data[(size_t)2 * l + kv].data()), bytes / 2);
        }
    DU_CUDA_TRY(cudaStreamSynchronize(m->stream));
    for (int l = 0; l < m->L; l++) {
        const SeqKv s = seq_kv(m, seq, l);
        DU_CUDA_TRY(cudaMemcpyAsync(s.k, data[(size_t)2 * l].data(), bytes, cudaMemcpyHostToDevice, m->stream));
        DU_CUDA_TRY(cudaMemcpyAsync(s.v, data[(size_t)2 * l + 1].data(), bytes, cudaMemcpyHostToDevice, m->stream));
    }
    m->h_cache_len[seq] = tokens;
    int rc = sync_cache_len(m);
    if (rc) return rc;
    DU_CUDA_TRY(cudaStreamSynchronize(m->stream));
    *loaded = 1;
    return DU_OK;
}

DU_API int du_model_save_kv(du_model *m, int seq, const char *path, uint64_t context_hash, const void *extra,
                            int extra_len)
{
    DU_GUARD(m);
    DU_CHECK_ARG(path && seq >= 0 && seq < m->maxb && extra_len >= 0 && (extra_len == 0 || extra),
                 "du_model_save_kv: bad arguments");
    const int tokens = m->h_cache_len[seq];
    if (tokens <= 0) return DU_OK;
    DU_CUDA_TRY(cudaStreamSynchronize(m->stream));
    std::vector<uint8_t> out;
    auto put = [&](const void *p, size_t n) {
        const uint8_t *b = static_cast<const uint8_t *>(p);
        out.insert(out.end(), b, b + n);
    };
    const uint8_t fmt = m->kv8 ? DU_KV_INT8 : DU_KV_FP16;
    put(&LMKV_MAGIC, 4);
    put(&LMKV_VERSION, 4);
    put(&context_hash, 8);
    put(&fmt, 1);
    put(&tokens, 4);
    put(&m->L, 4);
    put(&extra_len, 4);
    if (extra_len) put(extra, (size_t)extra_len);
    std::vector<uint8_t> buf;
    int rc = DU_OK;
    for (int l = 0; l < m->L; l++) {
        const SeqKv s = seq_kv(m, seq, l);
        const uint8_t kind = 0;
        put(&kind, 1);
        const void *src[4] = {s.k, s.v, s.ksz, s.vsz};
        const size_t len[4] = {(size_t)tokens * s.row_bytes, (size_t)tokens * s.row_bytes, (size_t)tokens * s.sz_bytes,
                               (size_t)tokens * s.sz_bytes};
        for (int b = 0; b < (m->kv8 ? 4 : 2); b++) {
            if ((rc = d2h(m, buf, src[b], len[b]))) return rc;
            DU_CUDA_TRY(cudaStreamSynchronize(m->stream));
            const int32_t n = (int32_t)buf.size();
            put(&n, 4);
            put(buf.data(), buf.size());
        }
    }
    return write_file(path, out.data(), out.size());
}

// Header of a du_model_save_kv file, without a model.  Returns DU_OK with *valid
// = 0 when the file is missing or is not such a snapshot.
DU_API int du_kv_file_peek(const char *path, int *valid, uint64_t *context_hash, int *kv_format, int *tokens,
                           int *layers, void *extra_out, int extra_cap, int *extra_len)
{
    DU_CHECK_ARG(path && valid, "du_kv_file_peek: null argument");
    *valid = 0;
    std::vector<uint8_t> f;
    if (!read_file(path, f) || f.size() < 29) return DU_OK;
    uint32_t magic;
    int32_t ver, tok, nl, xl;
    uint64_t hash;
    memcpy(&magic, f.data(), 4);
    memcpy(&ver, f.data() + 4, 4);
    memcpy(&hash, f.data() + 8, 8);
    const uint8_t fmt = f[16];
    memcpy(&tok, f.data() + 17, 4);
    memcpy(&nl, f.data() + 21, 4);
    memcpy(&xl, f.data() + 25, 4);
    if (magic != LMKV_MAGIC || ver != LMKV_VERSION || xl < 0 || (size_t)xl > f.size() - 29) return DU_OK;
    if (context_hash) *context_hash = hash;
    if (kv_format) *kv_format = fmt;
    if (tokens) *tokens = tok;
    if (layers) *layers = nl;
    if (extra_len) *extra_len = xl;
    if (extra_out && extra_cap >= xl && xl > 0) memcpy(extra_out, f.data() + 29, (size_t)xl);
    *valid = 1;
    return DU_OK;
}

DU_API int du_model_load_kv(du_model *m, int seq, const char *path, uint64_t expected_hash, int *loaded)
{
    DU_GUARD(m);
    DU_CHECK_ARG(path && loaded && seq >= 0 && seq < m->maxb, "du_model_load_kv: bad arguments");
    *loaded = 0;
    std::vector<uint8_t> f;
    if (!read_file(path, f) || f.size() < 29) return DU_OK;
    uint32_t magic;
    int32_t ver, tokens, nl, xl;
    uint64_t hash;
    memcpy(&magic, f.data(), 4);
    memcpy(&ver, f.data() + 4, 4);
    memcpy(&hash, f.data() + 8, 8);
    const uint8_t fmt = f[16];
    memcpy(&tokens, f.data() + 17, 4);
    memcpy(&nl, f.data() + 21, 4);
    memcpy(&xl, f.data() + 25, 4);
    if (magic != LMKV_MAGIC || ver != LMKV_VERSION || hash != expected_hash) return DU_OK;
    if (fmt != (m->kv8 ? DU_KV_INT8 : DU_KV_FP16) || nl != m->L || tokens <= 0 || tokens > m->cap) return DU_OK;
    if (xl < 0 || (size_t)xl > f.size() - 29) return DU_OK;
    // walk and check every blob before anything reaches the device
    size_t at = 29 + (size_t)xl;
    const int nb = m->kv8 ? 4 : 2;
    std::vector<size_t> offs;
    for (int l = 0; l < m->L; l++) {
        const SeqKv s = seq_kv(m, seq, l);
        if (at >= f.size() || f[at] != 0) return DU_OK;    // kind 0: full attention
        at++;
        for (int b = 0; b < nb; b++) {
            const size_t want = (size_t)tokens * (b < 2 ? s.row_bytes : s.sz_bytes);
            int32_t n;
            if (at + 4 > f.size()) return DU_OK;
            memcpy(&n, f.data() + at, 4);
            at += 4;
            if (n < 0 || (size_t)n != want || at + want > f.size()) return DU_OK;
            offs.push_back(at);
            at += want;
        }
    }
    if (at != f.size()) return DU_OK;
    DU_CUDA_TRY(cudaStreamSynchronize(m->stream));
    size_t i = 0;
    for (int l = 0; l < m->L; l++) {
        const SeqKv s = seq_kv(m, seq, l);
        uint8_t *dst[4] = {s.k, s.v, s.ksz, s.vsz};
        for (int b = 0; b < nb; b++, i++) {
            const size_t n = (size_t)tokens * (b < 2 ? s.row_bytes : s.sz_bytes);
            DU_CUDA_TRY(cudaMemcpyAsync(dst[b], f.data() + offs[i], n, cudaMemcpyHostToDevice, m->stream));
        }
    }
    m->h_cache_len[seq] = tokens;
    int rc = sync_cache_len(m);
    if (rc) return rc;
    DU_CUDA_TRY(cudaStreamSynchronize(m->stream));
    *loaded = 1;
    return DU_OK;
}

}  // extern "C"
