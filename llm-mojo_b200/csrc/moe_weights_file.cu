// The layer-blob weights file (gemma4_moe_weights_q4.bin): its layout, the
// MoE layer descriptor of a layer inside a loaded image, and a reader that
// streams a byte range of the file into HBM.
//
// Layout (model_speculative_moe_batched.mojo:57-231, written by
// convert_gemma4_moe.py:164-262): per layer, the packed Q4_0 bytes of
// q, k, v, o, gate, up, down, router, experts_gate_up, experts_down
// (each rows x cols / 2 bytes; v absent on global layers), then the fp32
// scales of the same matrices in the same order (rows x cols / 32 each),
// then twelve fp32 vectors (input_layernorm ... layer_scalar), the whole
// padded with zeros to a multiple of 4096 bytes.  Layer l starts at the sum
// of the padded sizes of layers 0..l-1.
//
// Reader: the reference reads the 14.3 GB file into host RAM in 256 MB
// chunks with one thread (:1366-1380) and the GPU then reads host memory.
// Here the bytes go to HBM once: the file range is cut into chunks of up to
// kChunk bytes; each chunk is read by kThreads host threads (pread on
// disjoint slices) into one of kBufs pinned buffers, and copied to the
// device with cudaMemcpyAsync on the caller's stream while the next chunk
// is being read.  A buffer is reused only after the event recorded behind
// its previous copy has completed.  The pinned buffers belong to the
// context and are kept between calls (pinning costs about as much as the
// copies of a small file).
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "moe_b200.h"
#include "moe_internal.h"

namespace {

constexpr int64_t kBlobAlign = 4096;

bool cfg_ok(const moe_model_config* c) {
    return c && c->embed_dim > 0 && c->standard_mlp_dim > 0 && c->expert_mlp_dim > 0 &&
           c->num_experts > 0 && c->top_k > 0 && c->num_layers > 0 && c->num_heads > 0 &&
           c->head_dim_sliding > 0 && c->kv_heads_sliding > 0 && c->head_dim_global > 0 &&
           c->kv_heads_global > 0 && c->global_every > 0;
}

// Fills everything but layer_offset.  Returns MOE_E_SHAPE when an inner
// dimension is not a positive multiple of 32.
int layout_in_blob(const moe_model_config* c, int64_t layer, moe_layer_layout* o) {
    std::memset(o, 0, sizeof(*o));
    const int64_t d = c->embed_dim, S = c->standard_mlp_dim, F = c->expert_mlp_dim,
                  E = c->num_experts, H = c->num_heads;
    const bool global = layer % c->global_every == c->global_every - 1;
    const int64_t hd = global ? c->head_dim_global : c->head_dim_sliding;
    const int64_t kv = global ? c->kv_heads_global : c->kv_heads_sliding;
    o->is_global = global;
    o->head_dim = hd;
    o->kv_heads = kv;
    // rows x cols (cols = inner dimension, the one Q4_0 blocks run along)
    const int64_t shape[MOE_W_COUNT][2] = {
        {H * hd, d},                       // q_proj
        {kv * hd, d},                      // k_proj
        {global ? 0 : kv * hd, d},         // v_proj (absent on global layers)
        {d, H * hd},                       // o_proj
        {S, d},                            // mlp.gate_proj
        {S, d},                            // mlp.up_proj
        {d, S},                            // mlp.down_proj
        {E, d},                            // router.proj
        {E * 2 * F, d},                    // experts.gate_up_proj, all experts stacked
        {E * d, F},                        // experts.down_proj, all experts stacked
    };
    for (int m = 0; m < MOE_W_COUNT; ++m) {
        o->rows[m] = shape[m][0];
        o->cols[m] = shape[m][1];
        if (o->cols[m] <= 0 || o->cols[m] % 32 != 0) return MOE_E_SHAPE;
    }
    int64_t off = 0;
    for (int m = 0; m < MOE_W_COUNT; ++m) {
        o->packed_offset[m] = off;
        off += o->rows[m] * o->cols[m] / 2;
    }
    for (int m = 0; m < MOE_W_COUNT; ++m) {
        o->scales_offset[m] = off;
        off += o->rows[m] * o->cols[m] / 32 * 4;
    }
    const int64_t vlen[MOE_V_COUNT] = {d, d, d, d, d, d, d, hd, hd, d, E, 1};
    for (int v = 0; v < MOE_V_COUNT; ++v) {
        o->vec_offset[v] = off;
        o->vec_len[v] = vlen[v];
        off += vlen[v] * 4;
    }
    o->payload_bytes = off;
    o->layer_bytes = (off + kBlobAlign - 1) / kBlobAlign * kBlobAlign;
    return MOE_OK;
}

// pread until `n` bytes are in.  Returns 0, the errno of a failed read, or
// EIO when the file ends early.
int read_full(int fd, char* dst, int64_t n, int64_t pos) {
    while (n > 0) {
        ssize_t r = pread(fd, dst, (size_t)std::min<int64_t>(n, 1 << 30), (off_t)pos);
        if (r < 0 && errno == EINTR) continue;
        if (r < 0) return errno;
        if (r == 0) return EIO;
        dst += r;
        n -= r;
        pos += r;
    }
    return 0;
}

}  // namespace

namespace moe {

void FileStaging::release() {
    for (cudaEvent_t e : ev)
        if (e) cudaEventDestroy(e);
    for (char* b : buf)
        if (b) cudaFreeHost(b);
    ev.clear();
    buf.clear();
    buf_bytes = 0;
}

int load_file_range(const char* path, int64_t file_offset, int64_t bytes, char* dst,
                    int64_t dst_capacity, cudaStream_t stream, FileStaging& st, std::string& err,
                    int64_t* loaded) {
    constexpr int64_t kChunk = 32ll << 20;  // largest staging buffer
    constexpr int kBufs = 4;
    const int kThreads = std::max(1u, std::min(8u, std::thread::hardware_concurrency()));
    *loaded = 0;
    int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) {
        err = std::string("cannot open ") + path + ": " + std::strerror(errno);
        return MOE_E_ARG;
    }
    struct stat sb;
    if (fstat(fd, &sb) != 0) {
        err = std::string("cannot stat ") + path + ": " + std::strerror(errno);
        close(fd);
        return MOE_E_ARG;
    }
    const int64_t size = sb.st_size;
    if (bytes < 0) bytes = size - file_offset;
    if (file_offset < 0 || bytes < 0 || file_offset + bytes > size) {
        err = std::string(path) + " holds " + std::to_string(size) + " bytes; requested [" +
              std::to_string(file_offset) + ", " + std::to_string(file_offset + bytes) + ")";
        close(fd);
        return MOE_E_SHAPE;
    }
    if (bytes > dst_capacity) {
        err = "the destination allocation holds " + std::to_string(dst_capacity) +
              " bytes from dst; the range is " + std::to_string(bytes);
        close(fd);
        return MOE_E_SHAPE;
    }
    if (bytes == 0) {
        close(fd);
        return MOE_OK;
    }
    posix_fadvise(fd, file_offset, bytes, POSIX_FADV_SEQUENTIAL);
    // staging: kBufs pinned buffers of up to kChunk bytes, grown on demand
    const int64_t want = std::min(kChunk, (bytes + (1 << 20) - 1) >> 20 << 20);
    int status = MOE_OK;
    auto cuda_err = [&](cudaError_t e, const char* where) {
        err = std::string(where) + ": " + cudaGetErrorString(e);
        status = MOE_E_CUDA;
    };
    if (st.buf_bytes < want) {
        st.release();
        st.buf.assign(kBufs, nullptr);
        st.ev.assign(kBufs, nullptr);
        for (int b = 0; b < kBufs && status == MOE_OK; ++b) {
            cudaError_t e = cudaHostAlloc((void**)&st.buf[b], (size_t)want, cudaHostAllocDefault);
            if (e != cudaSuccess) {
                cudaGetLastError();
                st.buf[b] = nullptr;
                err = "pinned staging allocation failed";
                status = MOE_E_NOMEM;
                break;
            }
            e = cudaEventCreateWithFlags(&st.ev[b], cudaEventDisableTiming);
            if (e != cudaSuccess) cuda_err(e, "cudaEventCreateWithFlags");
        }
        if (status != MOE_OK) {
            st.release();
            close(fd);
            return status;
        }
        st.buf_bytes = want;
    }
    const int64_t chunk_bytes = st.buf_bytes;
    std::vector<bool> in_flight(kBufs, false);
    int64_t done = 0;
    for (int64_t chunk = 0; status == MOE_OK && done < bytes; ++chunk) {
        const int b = (int)(chunk % kBufs);
        const int64_t n = std::min(chunk_bytes, bytes - done);
        if (in_flight[b]) {
            cudaError_t e = cudaEventSynchronize(st.ev[b]);
            if (e != cudaSuccess) {
                cuda_err(e, "cudaEventSynchronize");
                break;
            }
        }
        // disjoint slices of the chunk, 1 MiB-aligned, one per thread
        const int64_t slice = ((n + kThreads - 1) / kThreads + (1 << 20) - 1) >> 20 << 20;
        std::vector<std::thread> pool;
        std::vector<int> rc(kThreads, 0);
        for (int t = 0; t < kThreads; ++t) {
            const int64_t lo = t * slice, hi = std::min(n, lo + slice);
            if (lo >= hi) break;
            pool.emplace_back([&, t, lo, hi] {
                rc[t] = read_full(fd, st.buf[b] + lo, hi - lo, file_offset + done + lo);
            });
        }
        for (auto& th : pool) th.join();
        for (int t = 0; t < kThreads; ++t)
            if (rc[t] != 0) {
                err = std::string("read of ") + path + " failed at or after byte " +
                      std::to_string(file_offset + done + t * slice) + ": " + std::strerror(rc[t]);
                status = MOE_E_ARG;
                break;
            }
        if (status != MOE_OK) break;
        cudaError_t e = cudaMemcpyAsync(dst + done, st.buf[b], (size_t)n, cudaMemcpyHostToDevice, stream);
        if (e != cudaSuccess) {
            cuda_err(e, "cudaMemcpyAsync");
            break;
        }
        e = cudaEventRecord(st.ev[b], stream);
        if (e != cudaSuccess) {
            cuda_err(e, "cudaEventRecord");
            break;
        }
        in_flight[b] = true;
        done += n;
    }
    // every copy that was issued completes before the call returns, so the
    // buffers are idle between calls
    for (int b = 0; b < kBufs; ++b)
        if (in_flight[b]) {
            cudaError_t e = cudaEventSynchronize(st.ev[b]);
            if (e != cudaSuccess && status == MOE_OK) cuda_err(e, "cudaEventSynchronize");
        }
    close(fd);
    if (status == MOE_OK) *loaded = done;
    return status;
}

}  // namespace moe

extern "C" {

int moe_default_model_config(moe_model_config* c) {
    if (!c) return MOE_E_ARG;
    // MoEConfig defaults, model_speculative_moe_batched.mojo:41-50; the
    // attention shapes hard-coded in :59-63
    c->embed_dim = 2816;
    c->standard_mlp_dim = 2112;
    c->expert_mlp_dim = 704;
    c->num_experts = 128;
    c->top_k = 8;
    c->num_layers = 30;
    c->num_heads = 16;
    c->head_dim_sliding = 256;
    c->kv_heads_sliding = 8;
    c->head_dim_global = 512;
    c->kv_heads_global = 2;
    c->global_every = 6;
    return MOE_OK;
}

int moe_weights_layout(const moe_model_config* c, int64_t layer, moe_layer_layout* out) {
    if (!out || !cfg_ok(c)) return MOE_E_ARG;
    if (layer < 0 || layer >= c->num_layers) return MOE_E_ARG;
    int64_t off = 0;
    moe_layer_layout tmp;
    for (int64_t l = 0; l < layer; ++l) {
        int s = layout_in_blob(c, l, &tmp);
        if (s != MOE_OK) return s;
        off += tmp.layer_bytes;
    }
    int s = layout_in_blob(c, layer, out);
    if (s != MOE_OK) return s;
    out->layer_offset = off;
    return MOE_OK;
}

int moe_weights_file_size(const moe_model_config* c, int64_t* bytes) {
    if (!bytes || !cfg_ok(c)) return MOE_E_ARG;
    moe_layer_layout last;
    int s = moe_weights_layout(c, c->num_layers - 1, &last);
    if (s != MOE_OK) return s;
    *bytes = last.layer_offset + last.layer_bytes;
    return MOE_OK;
}

int moe_layer_desc_from_weights(const moe_model_config* c, const void* weights_base, int64_t layer,
                                moe_layer_desc* out) {
    if (!out || !weights_base || !cfg_ok(c)) return MOE_E_ARG;
    if (c->num_experts > 1024 || c->top_k > 32 || c->top_k > c->num_experts) return MOE_E_SHAPE;
    moe_layer_layout L;
    int s = moe_weights_layout(c, layer, &L);
    if (s != MOE_OK) return s;
    const char* b = static_cast<const char*>(weights_base) + L.layer_offset;
    std::memset(out, 0, sizeof(*out));
    out->embed_dim = c->embed_dim;
    out->expert_mlp_dim = c->expert_mlp_dim;
    out->num_experts = c->num_experts;
    out->top_k = c->top_k;
    out->activation = MOE_ACT_SIGMOID1702;
    // Float32(1.0 / sqrt(Float32(embed_dim))), model_speculative_moe_batched.mojo:1867
    out->r_scale_factor = 1.0f / std::sqrt((float)c->embed_dim);
    out->moe_top_p = 1.0f;
    out->router_packed = reinterpret_cast<const uint8_t*>(b + L.packed_offset[MOE_W_ROUTER]);
    out->router_scales = reinterpret_cast<const float*>(b + L.scales_offset[MOE_W_ROUTER]);
    out->router_scale = reinterpret_cast<const float*>(b + L.vec_offset[MOE_V_ROUTER_SCALE]);
    out->per_expert_scale =
        reinterpret_cast<const float*>(b + L.vec_offset[MOE_V_ROUTER_PER_EXPERT_SCALE]);
    out->pre_norm_w = reinterpret_cast<const float*>(b + L.vec_offset[MOE_V_PRE_FEEDFORWARD_LAYERNORM_2]);
    out->post_norm_w =
        reinterpret_cast<const float*>(b + L.vec_offset[MOE_V_POST_FEEDFORWARD_LAYERNORM_2]);
    out->gate_up_packed = reinterpret_cast<const uint8_t*>(b + L.packed_offset[MOE_W_EXPERTS_GATE_UP]);
    out->gate_up_scales = reinterpret_cast<const float*>(b + L.scales_offset[MOE_W_EXPERTS_GATE_UP]);
    out->down_packed = reinterpret_cast<const uint8_t*>(b + L.packed_offset[MOE_W_EXPERTS_DOWN]);
    out->down_scales = reinterpret_cast<const float*>(b + L.scales_offset[MOE_W_EXPERTS_DOWN]);
    return MOE_OK;
}

}  // extern "C"
