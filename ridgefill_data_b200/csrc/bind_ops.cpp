// Python bindings of the non-GEMM kernels (kernels.h). Tensors are checked for device, dtype and the
// contiguity each kernel assumes; strides that kernels take explicitly are passed from Python.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "kernels.h"

torch::Tensor& err_word(int dev);   // bindings.cpp: the per-device error word

namespace {

using at::Tensor;
using OptT = c10::optional<Tensor>;

cudaStream_t cur() { return at::cuda::getCurrentCUDAStream().stream(); }
const __nv_bfloat16* cbf(const Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); }
__nv_bfloat16* bf(const Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }

void need(const Tensor& t, at::ScalarType st, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == st, name, " has dtype ", t.scalar_type(), ", expected ", st);
}

void rmsnorm(Tensor x, Tensor w, Tensor out, double eps, bool zero_centred) {
  need(x, at::kBFloat16, "x");
  need(w, at::kBFloat16, "w");
  need(out, at::kBFloat16, "out");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && out.stride(1) == 1, "rmsnorm: 2-D rows");
  const int d = (int)x.size(1);
  TORCH_CHECK(d % 8 == 0 && d <= 8192 && w.numel() == d, "rmsnorm: d % 8 == 0, d <= 8192");
  TORCH_CHECK(x.stride(0) % 8 == 0 && out.stride(0) % 8 == 0, "rmsnorm: row pitch % 8");
  c10::cuda::CUDAGuard g(x.device());
  rf::rmsnorm(cbf(x), x.stride(0), cbf(w), bf(out), out.stride(0), (int)x.size(0), d, (float)eps, zero_centred ? 1 : 0,
              cur());
}

void head_norm_rope(Tensor src, int64_t src_row_stride, int64_t src_head_stride, int64_t n_heads, int64_t head_dim,
                    int64_t n_rows, OptT norm_w, int64_t norm_mode, double eps, OptT cos, OptT sin, int64_t rot,
                    OptT pos, int64_t pos_offset, Tensor dst, int64_t dst_head_stride, int64_t dst_row_stride,
                    OptT dst_pages, int64_t page_size, int64_t dst_page_stride, int64_t dst_row0,
                    bool dst_row_from_pos, int64_t dst_rows) {
  need(src, at::kBFloat16, "src");
  need(dst, at::kBFloat16, "dst");
  TORCH_CHECK(head_dim % 32 == 0 && head_dim <= 256, "head_norm_rope: head_dim % 32 == 0, <= 256");
  TORCH_CHECK(rot == 0 || ((rot / 2) % (head_dim / 32) == 0 && rot <= head_dim), "head_norm_rope: rot layout");
  c10::cuda::CUDAGuard g(src.device());
  rf::HeadNormRopeArgs a{};
  a.src = cbf(src);
  a.src_row_stride = src_row_stride;
  a.src_head_stride = src_head_stride;
  a.n_heads = (int)n_heads;
  a.head_dim = (int)head_dim;
  a.n_rows = (int)n_rows;
  a.norm_w = norm_w.has_value() ? cbf(*norm_w) : nullptr;
  a.norm_mode = norm_w.has_value() ? (int)norm_mode : -1;
  a.eps = (float)eps;
  a.rot = (int)rot;
  if (rot > 0) {
    TORCH_CHECK(cos.has_value() && sin.has_value(), "head_norm_rope: cos/sin tables");
    need(*cos, at::kBFloat16, "cos");
    a.cos = cbf(*cos);
    a.sin = cbf(*sin);
  }
  if (pos.has_value()) {
    need(*pos, at::kInt, "pos");
    a.pos = pos->data_ptr<int>();
  }
  a.pos_offset = (int)pos_offset;
  if (dst_pages.has_value()) {
    need(*dst_pages, at::kInt, "dst_pages");
    TORCH_CHECK(page_size > 0, "head_norm_rope: page_size");
    a.dst_pages = dst_pages->data_ptr<int>();
    a.page_size = (int)page_size;
    a.dst_page_stride = dst_page_stride;
    a.dst_row0 = (int)dst_row0;
  }
  if (dst_row_from_pos) {
    TORCH_CHECK(pos.has_value() && dst_rows > 0, "head_norm_rope: rows from positions need pos and the capacity");
    a.dst_row_from_pos = 1;
    a.dst_rows = (int)dst_rows;
  }
  a.dst = bf(dst);
  a.dst_head_stride = dst_head_stride;
  a.dst_row_stride = dst_row_stride;
  rf::head_norm_rope(a, cur());
}

void gated_rmsnorm(Tensor o, Tensor z, int64_t ldz, Tensor w, Tensor out, int64_t heads, int64_t dv, double eps) {
  need(o, at::kBFloat16, "o");
  need(z, at::kBFloat16, "z");
  need(w, at::kBFloat16, "w");
  need(out, at::kBFloat16, "out");
  TORCH_CHECK(dv % 32 == 0 && dv <= 256, "gated_rmsnorm: dv");
  c10::cuda::CUDAGuard g(o.device());
  rf::gated_rmsnorm(cbf(o), o.stride(0), cbf(z), ldz, cbf(w), bf(out), out.stride(0), (int)o.size(0), (int)heads,
                    (int)dv, (float)eps, cur());
}

void embed_gather(Tensor table, Tensor ids, Tensor out) {
  need(table, at::kBFloat16, "table");
  need(ids, at::kLong, "ids");
  need(out, at::kBFloat16, "out");
  TORCH_CHECK(table.is_contiguous() && out.is_contiguous() && ids.is_contiguous(), "embed_gather: contiguous");
  TORCH_CHECK(table.size(1) % 8 == 0, "embed_gather: d % 8");
  c10::cuda::CUDAGuard g(table.device());
  rf::embed_gather(cbf(table), ids.data_ptr<int64_t>(), bf(out), (int)ids.numel(), (int)table.size(1),
                   (long)table.size(0), cur(), err_word(table.device().index()).data_ptr<int>());
}

void flash_attention(Tensor q, int64_t q_head_stride, Tensor k, Tensor v, int64_t kv_head_stride, Tensor out,
                     int64_t hq, int64_t hkv, int64_t hd, int64_t nq, int64_t nk, OptT qpos, int64_t q_start,
                     double scale, OptT gate, int64_t gate_row, int64_t gate_head, int64_t impl, Tensor err,
                     OptT kv_pages, int64_t page_size, int64_t num_pages) {
  need(q, at::kBFloat16, "q");
  need(k, at::kBFloat16, "k");
  need(v, at::kBFloat16, "v");
  need(out, at::kBFloat16, "out");
  TORCH_CHECK(hd == 64 || hd == 128 || hd == 256, "flash_attention: head_dim 64/128/256");
  TORCH_CHECK(hq % hkv == 0, "flash_attention: GQA");
  TORCH_CHECK(out.stride(1) == 1, "flash_attention: out rows");
  c10::cuda::CUDAGuard g(q.device());
  rf::AttnArgs a{};
  a.q = cbf(q);
  a.q_head_stride = q_head_stride;
  a.k = cbf(k);
  a.v = cbf(v);
  a.kv_head_stride = kv_head_stride;
  a.hq = (int)hq;
  a.hkv = (int)hkv;
  a.hd = (int)hd;
  a.nq = (int)nq;
  a.nk = (int)nk;
  if (qpos.has_value()) {
    need(*qpos, at::kInt, "qpos");
    a.qpos = qpos->data_ptr<int>();
  }
  a.q_start = (int)q_start;
  a.scale = (float)scale;
  if (gate.has_value()) {
    need(*gate, at::kBFloat16, "gate");
    a.gate = cbf(*gate);
    a.gate_row = gate_row;
    a.gate_head = gate_head;
  }
  a.out = bf(out);
  a.out_row = out.stride(0);
  a.err = err.data_ptr<int>();
  a.impl = (int)impl;
  if (kv_pages.has_value()) {
    need(*kv_pages, at::kInt, "kv_pages");
    a.kv_pages = kv_pages->data_ptr<int>();
    a.page_size = (int)page_size;
    a.num_pages = (int)num_pages;
    TORCH_CHECK(kv_pages->numel() * page_size >= nk, "flash_attention: the page table covers fewer than nk rows");
  }
  rf::flash_attention(a, cur());
}

void gdn_prep(Tensor proj, int64_t b_off, int64_t a_off, Tensor conv_w, OptT conv_state, Tensor A_log,
              Tensor dt_bias, int64_t n, int64_t nk, int64_t nv, int64_t dk, int64_t dv, int64_t K, OptT q, Tensor k,
              Tensor v, Tensor beta, Tensor g) {
  need(proj, at::kBFloat16, "proj");
  need(conv_w, at::kBFloat16, "conv_w");
  need(A_log, at::kFloat, "A_log");
  need(dt_bias, at::kFloat, "dt_bias");
  if (q.has_value()) need(*q, at::kBFloat16, "q");
  need(k, at::kBFloat16, "k");
  need(v, at::kBFloat16, "v");
  need(beta, at::kFloat, "beta");
  need(g, at::kFloat, "g");
  TORCH_CHECK(proj.stride(1) == 1 && conv_w.is_contiguous(), "gdn_prep: layouts");
  TORCH_CHECK(dk % 32 == 0 && dv % 32 == 0 && dk <= 128 && dv <= 128 && K <= 8, "gdn_prep: dims");
  c10::cuda::CUDAGuard gd(proj.device());
  rf::GdnPrepArgs a{};
  a.proj = cbf(proj);
  a.proj_row = proj.stride(0);
  a.b_off = (int)b_off;
  a.a_off = (int)a_off;
  a.conv_w = cbf(conv_w);
  if (conv_state.has_value()) {
    need(*conv_state, at::kBFloat16, "conv_state");
    a.conv_state = cbf(*conv_state);
  }
  a.A_log = A_log.data_ptr<float>();
  a.dt_bias = dt_bias.data_ptr<float>();
  a.n = (int)n;
  a.nk = (int)nk;
  a.nv = (int)nv;
  a.dk = (int)dk;
  a.dv = (int)dv;
  a.K = (int)K;
  a.q = q.has_value() ? bf(*q) : nullptr;
  a.k = bf(k);
  a.v = bf(v);
  a.beta = beta.data_ptr<float>();
  a.g = g.data_ptr<float>();
  rf::gdn_prep(a, cur());
}

void gdn_conv_state_update(Tensor proj, Tensor state, int64_t n, int64_t C, int64_t K) {
  need(proj, at::kBFloat16, "proj");
  need(state, at::kBFloat16, "state");
  TORCH_CHECK(state.is_contiguous() && K <= 8, "gdn_conv_state_update: layout");
  c10::cuda::CUDAGuard g(proj.device());
  rf::gdn_conv_state_update(cbf(proj), proj.stride(0), bf(state), (int)n, (int)C, (int)K, cur());
}

// One decode row of a GDN layer for R sequences: proj [R, *] (rows of the in-projection), out [R, nv * dv]; the
// per-sequence conv states [K-1, C] bf16 and recurrent states [nv, dk, dv] fp32 are read from *_src and written to
// *_dst (the same tensors: in place).
void gdn_decode_step(Tensor proj, Tensor conv_w, Tensor A_log, Tensor dt_bias, std::vector<Tensor> conv_src,
                     std::vector<Tensor> conv_dst, std::vector<Tensor> rec_src, std::vector<Tensor> rec_dst, Tensor out,
                     int64_t b_off, int64_t a_off, int64_t nk, int64_t nv, int64_t dk, int64_t dv, int64_t K) {
  need(proj, at::kBFloat16, "proj");
  need(conv_w, at::kBFloat16, "conv_w");
  need(A_log, at::kFloat, "A_log");
  need(dt_bias, at::kFloat, "dt_bias");
  need(out, at::kBFloat16, "out");
  const int64_t R = proj.size(0);
  const int64_t C = 2 * nk * dk + nv * dv;
  TORCH_CHECK(rf::gdn_decode_supported((int)dk, (int)dv, (int)K) && nk > 0 && nv % nk == 0,
              "gdn_decode_step: dims");
  TORCH_CHECK(proj.stride(1) == 1 && out.stride(1) == 1 && conv_w.is_contiguous() && out.size(0) == R &&
                  out.size(1) == nv * dv && proj.size(1) >= a_off + nv && b_off + nv <= a_off && C <= b_off &&
                  conv_w.size(0) == C && conv_w.size(1) == K && A_log.numel() == nv && dt_bias.numel() == nv,
              "gdn_decode_step: layouts");
  TORCH_CHECK((int64_t)conv_src.size() == R && (int64_t)conv_dst.size() == R && (int64_t)rec_src.size() == R &&
                  (int64_t)rec_dst.size() == R, "gdn_decode_step: one state of each kind per row");
  for (int64_t r = 0; r < R; ++r) {
    for (const Tensor* t : {&conv_src[r], &conv_dst[r]}) {
      need(*t, at::kBFloat16, "conv state");
      TORCH_CHECK(t->is_contiguous() && t->numel() == (K - 1) * C && t->device() == proj.device(),
                  "gdn_decode_step: conv state [K-1, C]");
    }
    for (const Tensor* t : {&rec_src[r], &rec_dst[r]}) {
      need(*t, at::kFloat, "recurrent state");
      TORCH_CHECK(t->is_contiguous() && t->numel() == nv * dk * dv && t->device() == proj.device(),
                  "gdn_decode_step: recurrent state [nv, dk, dv]");
    }
  }
  c10::cuda::CUDAGuard gd(proj.device());
  for (int64_t r0 = 0; r0 < R; r0 += rf::kDecodeSeqs) {
    const int rows = (int)std::min<int64_t>(rf::kDecodeSeqs, R - r0);
    rf::GdnDecodeArgs a{};
    a.proj = cbf(proj);
    a.proj_row = proj.stride(0);
    a.b_off = (int)b_off;
    a.a_off = (int)a_off;
    a.conv_w = cbf(conv_w);
    a.A_log = A_log.data_ptr<float>();
    a.dt_bias = dt_bias.data_ptr<float>();
    a.nk = (int)nk;
    a.nv = (int)nv;
    a.dk = (int)dk;
    a.dv = (int)dv;
    a.K = (int)K;
    a.out = bf(out);
    a.out_row = out.stride(0);
    for (int s = 0; s < rows; ++s) {
      a.conv_src[s] = cbf(conv_src[r0 + s]);
      a.conv_dst[s] = bf(conv_dst[r0 + s]);
      a.rec_src[s] = rec_src[r0 + s].data_ptr<float>();
      a.rec_dst[s] = rec_dst[r0 + s].data_ptr<float>();
    }
    rf::gdn_decode_step(a, (int)r0, rows, cur());
  }
}

// One decode row of an attention layer for R sequences (attention_decode.cu). k / v: per sequence, its contiguous
// [hkv, rows, hd] buffers or the pool's K / V tensors; pages: empty (contiguous) or one int32 page table per
// sequence; rows / head_stride per sequence; part_o / part_ml the split workspace.
void decode_attention(Tensor qkv, Tensor pos, std::vector<Tensor> k, std::vector<Tensor> v, std::vector<Tensor> pages,
                      std::vector<int64_t> rows, std::vector<int64_t> head_stride, int64_t page_size,
                      int64_t page_stride, OptT q_norm, OptT k_norm, int64_t norm_mode, double eps, OptT cos, OptT sin,
                      int64_t rot, double scale, int64_t hq, int64_t hkv, int64_t hd, bool gated, Tensor out,
                      Tensor part_o, Tensor part_ml, Tensor err) {
  need(qkv, at::kBFloat16, "qkv");
  need(pos, at::kInt, "pos");
  need(out, at::kBFloat16, "out");
  need(part_o, at::kFloat, "part_o");
  need(part_ml, at::kFloat, "part_ml");
  need(err, at::kInt, "err");
  const int64_t R = qkv.size(0);
  TORCH_CHECK(rf::decode_attention_supported((int)hd, (int)hq, (int)hkv, (int)rot), "decode_attention: dims");
  const int64_t G = hq / hkv;
  const int64_t qw = hq * hd * (gated ? 2 : 1);
  TORCH_CHECK(qkv.stride(1) == 1 && qkv.size(1) >= qw + 2 * hkv * hd && pos.is_contiguous() && pos.numel() == R &&
                  out.stride(1) == 1 && out.size(0) == R && out.size(1) == hq * hd,
              "decode_attention: layouts");
  const int64_t S = rf::kDecSplits;
  TORCH_CHECK(part_o.numel() >= R * hkv * S * G * hd && part_ml.numel() >= R * hkv * S * G * 2,
              "decode_attention: workspace");
  TORCH_CHECK((int64_t)k.size() == R && (int64_t)v.size() == R && (int64_t)rows.size() == R &&
                  (int64_t)head_stride.size() == R && (pages.empty() || (int64_t)pages.size() == R),
              "decode_attention: one cache per row");
  TORCH_CHECK(rot == 0 || (cos.has_value() && sin.has_value()), "decode_attention: RoPE tables");
  // rows are read in hd / 32-element vectors (up to 16 bytes): 16-byte aligned bases and row pitches
  auto aligned = [](const Tensor& t) { return reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0; };
  TORCH_CHECK(aligned(qkv) && qkv.stride(0) % 8 == 0, "decode_attention: qkv alignment");
  TORCH_CHECK((!q_norm.has_value() || aligned(*q_norm)) && (!k_norm.has_value() || aligned(*k_norm)),
              "decode_attention: norm weight alignment");
  TORCH_CHECK(norm_mode < 0 || (q_norm.has_value() && k_norm.has_value()), "decode_attention: norm weights");
  for (int64_t r = 0; r < R; ++r) {
    TORCH_CHECK(rows[r] > 0, "decode_attention: empty cache");
    for (const Tensor* t : {&k[r], &v[r]}) {
      need(*t, at::kBFloat16, "cache");
      TORCH_CHECK(t->is_contiguous() && t->device() == qkv.device() && aligned(*t), "decode_attention: cache layout");
    }
    if (pages.empty()) {
      TORCH_CHECK(head_stride[r] >= rows[r] * hd && k[r].numel() >= hkv * head_stride[r] &&
                      v[r].numel() >= hkv * head_stride[r], "decode_attention: contiguous cache extent");
    } else {
      need(pages[r], at::kInt, "pages");
      TORCH_CHECK(page_size > 0 && pages[r].numel() * page_size >= rows[r] && head_stride[r] == page_size * hd &&
                      page_stride >= hkv * page_size * hd, "decode_attention: page table");
    }
  }
  c10::cuda::CUDAGuard gd(qkv.device());
  for (int64_t r0 = 0; r0 < R; r0 += rf::kDecodeSeqs) {
    const int n = (int)std::min<int64_t>(rf::kDecodeSeqs, R - r0);
    rf::DecodeAttnArgs a{};
    a.qkv = cbf(qkv);
    a.qkv_row = qkv.stride(0);
    a.hq = (int)hq;
    a.hkv = (int)hkv;
    a.hd = (int)hd;
    a.gated = gated ? 1 : 0;
    a.q_norm = q_norm.has_value() ? cbf(*q_norm) : nullptr;
    a.k_norm = k_norm.has_value() ? cbf(*k_norm) : nullptr;
    a.norm_mode = (int)norm_mode;
    a.eps = (float)eps;
    a.cos = cos.has_value() ? cbf(*cos) : nullptr;
    a.sin = sin.has_value() ? cbf(*sin) : nullptr;
    a.rot = (int)rot;
    a.pos = pos.data_ptr<int>();
    a.scale_log2 = (float)(scale * 1.4426950408889634);
    a.out = bf(out);
    a.out_row = out.stride(0);
    a.part_o = part_o.data_ptr<float>();
    a.part_ml = part_ml.data_ptr<float>();
    a.err = err.data_ptr<int>();
    a.page_size = (int)page_size;
    a.page_stride = page_stride;
    for (int s = 0; s < n; ++s) {
      a.k[s] = bf(k[r0 + s]);
      a.v[s] = bf(v[r0 + s]);
      a.pages[s] = pages.empty() ? nullptr : pages[r0 + s].data_ptr<int>();
      a.rows[s] = (int)rows[r0 + s];
      a.head_stride[s] = head_stride[r0 + s];
    }
    rf::decode_attention(a, (int)r0, n, cur());
  }
}

void gdn_chunk_scan(OptT q, Tensor k, Tensor v, Tensor beta, Tensor g, Tensor state, OptT out, Tensor w_buf,
                    Tensor u_buf, OptT s_buf, OptT vt_buf, int64_t n, int64_t nk, int64_t nv, int64_t dk, int64_t dv, Tensor err,
                    int64_t groups, OptT grp_buf, OptT start_buf) {
  need(k, at::kBFloat16, "k");
  need(v, at::kBFloat16, "v");
  need(beta, at::kFloat, "beta");
  need(g, at::kFloat, "g");
  need(state, at::kFloat, "state");
  need(w_buf, at::kBFloat16, "w_buf");
  need(u_buf, at::kBFloat16, "u_buf");
  TORCH_CHECK(dk == 128 && dv % 64 == 0 && dv <= 128 && nv % nk == 0, "gdn_chunk_scan: dk 128, dv 64 | 128");
  const int64_t n_pad = (n + 63) / 64 * 64;
  TORCH_CHECK(w_buf.numel() >= nv * n_pad * dk && u_buf.numel() >= nv * n_pad * dv, "gdn_chunk_scan: scratch size");
  TORCH_CHECK(state.is_contiguous() && state.numel() == nv * dk * dv, "gdn_chunk_scan: state [nv, dk, dv]");
  c10::cuda::CUDAGuard gd(k.device());
  rf::GdnScanArgs a{};
  if (q.has_value()) {
    need(*q, at::kBFloat16, "q");
    a.q = cbf(*q);
    TORCH_CHECK(out.has_value(), "gdn_chunk_scan: output mode needs out");
    // s_buf / vt_buf: only the split output path (gdn_fused_output = 0) reads them
    TORCH_CHECK(rf::gdn_fused_output || (s_buf.has_value() && vt_buf.has_value()),
                "gdn_chunk_scan: the split output path needs s_buf and vt_buf");
    if (s_buf.has_value() && vt_buf.has_value()) {
      need(*s_buf, at::kBFloat16, "s_buf");
      need(*vt_buf, at::kBFloat16, "vt_buf");
      TORCH_CHECK(s_buf->numel() >= nv * (n_pad / 64) * dk * dv, "gdn_chunk_scan: s_buf size");
      TORCH_CHECK(vt_buf->numel() >= nv * n_pad * dv, "gdn_chunk_scan: vt_buf size");
      a.s_buf = bf(*s_buf);
      a.vt_buf = bf(*vt_buf);
    }
  }
  a.k = cbf(k);
  a.v = cbf(v);
  a.beta = beta.data_ptr<float>();
  a.g = g.data_ptr<float>();
  a.state = state.data_ptr<float>();
  if (out.has_value()) {
    need(*out, at::kBFloat16, "out");
    a.out = bf(*out);
    a.out_row = out->stride(0);
  }
  a.w_buf = bf(w_buf);
  a.u_buf = bf(u_buf);
  a.n = (int)n;
  a.nk = (int)nk;
  a.nv = (int)nv;
  a.dk = (int)dk;
  a.dv = (int)dv;
  a.err = err.data_ptr<int>();
  if (groups > 1 && grp_buf.has_value()) {
    need(*grp_buf, at::kFloat, "grp_buf");
    TORCH_CHECK(grp_buf->numel() >= 2 * nv * groups * dv * dk, "gdn_chunk_scan: grp_buf size");
    a.groups = (int)groups;
    a.grp_buf = grp_buf->data_ptr<float>();
    if (start_buf.has_value()) {
      need(*start_buf, at::kFloat, "start_buf");
      TORCH_CHECK(start_buf->numel() >= nv * groups * dv * dk, "gdn_chunk_scan: start_buf size");
      a.start_buf = start_buf->data_ptr<float>();
    }
  }
  rf::gdn_chunk_scan(a, cur());
}

}  // namespace

void register_ops(pybind11::module_& m) {
  namespace py = pybind11;
  m.def("rmsnorm", &rmsnorm);
  m.def("head_norm_rope", &head_norm_rope, py::arg("src"), py::arg("src_row_stride"), py::arg("src_head_stride"),
        py::arg("n_heads"), py::arg("head_dim"), py::arg("n_rows"), py::arg("norm_w"), py::arg("norm_mode"),
        py::arg("eps"), py::arg("cos"), py::arg("sin"), py::arg("rot"), py::arg("pos"), py::arg("pos_offset"),
        py::arg("dst"), py::arg("dst_head_stride"), py::arg("dst_row_stride"), py::arg("dst_pages") = py::none(),
        py::arg("page_size") = 0, py::arg("dst_page_stride") = 0, py::arg("dst_row0") = 0,
        py::arg("dst_row_from_pos") = false, py::arg("dst_rows") = 0);
  m.def("gated_rmsnorm", &gated_rmsnorm);
  m.def("embed_gather", &embed_gather);
  m.def("flash_attention", &flash_attention, py::arg("q"), py::arg("q_head_stride"), py::arg("k"), py::arg("v"),
        py::arg("kv_head_stride"), py::arg("out"), py::arg("hq"), py::arg("hkv"), py::arg("hd"), py::arg("nq"),
        py::arg("nk"), py::arg("qpos"), py::arg("q_start"), py::arg("scale"), py::arg("gate"), py::arg("gate_row"),
        py::arg("gate_head"), py::arg("impl"), py::arg("err"), py::arg("kv_pages") = py::none(),
        py::arg("page_size") = 0, py::arg("num_pages") = 0);
  m.def("gdn_prep", &gdn_prep);
  m.def("gdn_conv_state_update", &gdn_conv_state_update);
  m.def("gdn_decode_step", &gdn_decode_step);
  m.def("decode_attention", &decode_attention);
  m.def("gdn_chunk_scan", &gdn_chunk_scan);
  void register_comm(pybind11::module_ & m);
  register_comm(m);
}

// ---------------------------------------------------------------------------------- comm bindings
#include "gemm.h"

namespace {

int64_t ipc_malloc_b(int64_t bytes) { return reinterpret_cast<int64_t>(rf::ipc_malloc((size_t)bytes)); }
void ipc_free_b(int64_t p) { rf::ipc_free(reinterpret_cast<void*>(p)); }
pybind11::bytes ipc_handle_b(int64_t p) { return pybind11::bytes(rf::ipc_handle(reinterpret_cast<void*>(p))); }
int64_t ipc_open_b(pybind11::bytes h) { return reinterpret_cast<int64_t>(rf::ipc_open(std::string(h))); }
void ipc_close_b(int64_t p) { rf::ipc_close(reinterpret_cast<void*>(p)); }

// A non-owning tensor view of device memory at `ptr`.
Tensor tensor_at(int64_t ptr, std::vector<int64_t> shape, int64_t dtype_code, int64_t device) {
  const at::ScalarType st = dtype_code == 0 ? at::kBFloat16 : dtype_code == 1 ? at::kFloat : dtype_code == 2 ? at::kInt
                                                                                                            : at::kDouble;
  return torch::from_blob(reinterpret_cast<void*>(ptr), shape,
                          torch::TensorOptions().dtype(st).device(torch::kCUDA, (int)device));
}

rf::PeerFlags flags_of(const std::vector<int64_t>& ptrs) {
  rf::PeerFlags f{};
  TORCH_CHECK(ptrs.size() <= rf::kMaxRanks, "at most 8 ranks");
  f.n = (int)ptrs.size();
  for (size_t i = 0; i < ptrs.size(); ++i) f.ptr[i] = reinterpret_cast<int*>(ptrs[i]);
  return f;
}

void comm_signal_b(std::vector<int64_t> flag_ptrs, int64_t slot, int64_t value) {
  rf::comm_signal(flags_of(flag_ptrs), (int)slot, (int)value, cur());
}

void comm_wait_b(int64_t flags, int64_t first, int64_t n, int64_t value, Tensor err, int64_t limit_ns) {
  rf::comm_wait(reinterpret_cast<const int*>(flags), (int)first, (int)n, (int)value, err.data_ptr<int>(), cur(),
                (uint64_t)std::max<int64_t>(0, limit_ns));
}

void comm_reduce_rows_b(int64_t recv, int64_t slot_stride, c10::optional<Tensor> residual, int64_t red, int64_t rows,
                        int64_t d, int64_t n_peers, int64_t my_rank, int64_t flags, int64_t arrive_slot,
                        int64_t reduced_slot, int64_t value, int64_t counter, std::vector<int64_t> peer_flags,
                        Tensor err) {
  rf::ReduceRowsArgs a{};
  a.recv = reinterpret_cast<const __nv_bfloat16*>(recv);
  a.slot_stride = slot_stride;
  if (residual.has_value()) {
    need(*residual, at::kBFloat16, "residual");
    a.residual = cbf(*residual);
    a.ld_res = residual->stride(0);
  }
  a.red = reinterpret_cast<__nv_bfloat16*>(red);
  a.rows = (int)rows;
  a.d = (int)d;
  a.n_peers = (int)n_peers;
  a.my_rank = (int)my_rank;
  a.flags = reinterpret_cast<const int*>(flags);
  a.arrive_slot = (int)arrive_slot;
  a.reduced_slot = (int)reduced_slot;
  a.value = (int)value;
  a.counter = reinterpret_cast<int*>(counter);
  a.peer_flags = flags_of(peer_flags);
  a.err = err.data_ptr<int>();
  TORCH_CHECK(d % 8 == 0, "comm_reduce_rows: d % 8");
  rf::comm_reduce_rows(a, cur());
}

void comm_gather_rows_b(std::vector<int64_t> peer_red, int64_t row_chunk, int64_t total_rows, int64_t d, Tensor out,
                        int64_t flags, int64_t reduced_slot, int64_t value, Tensor err) {
  need(out, at::kBFloat16, "out");
  rf::GatherRowsArgs a{};
  TORCH_CHECK(peer_red.size() <= rf::kMaxRanks, "at most 8 ranks");
  for (size_t i = 0; i < peer_red.size(); ++i) a.peer_red[i] = reinterpret_cast<const __nv_bfloat16*>(peer_red[i]);
  a.n_peers = (int)peer_red.size();
  a.row_chunk = (int)row_chunk;
  a.total_rows = (int)total_rows;
  a.d = (int)d;
  a.out = bf(out);
  a.ld_out = out.stride(0);
  a.flags = reinterpret_cast<const int*>(flags);
  a.reduced_slot = (int)reduced_slot;
  a.value = (int)value;
  a.err = err.data_ptr<int>();
  rf::comm_gather_rows(a, cur());
}

// tcgen05 GEMM whose epilogue stores bf16 tiles into peer buffers (gemm.h: PeerArgs).
void gemm_peer_b(Tensor a, Tensor b, c10::optional<Tensor> bias, std::vector<int64_t> peers, int64_t mode,
                 int64_t slot, int64_t row_chunk, int64_t slot_stride, int64_t ld, int64_t col_off, int64_t bn,
                 Tensor err) {
  need(a, at::kBFloat16, "a");
  need(b, at::kBFloat16, "b");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1, "gemm_peer: unit inner stride");
  TORCH_CHECK(peers.size() >= 1 && peers.size() <= rf::kMaxPeers, "gemm_peer: 1..8 peers");
  c10::cuda::CUDAGuard g(a.device());
  rf::GemmOperands op{a.data_ptr(), a.stride(0), false, b.data_ptr(), b.stride(0), false};
  rf::GemmArgs args{};
  args.M = (int)a.size(0);
  args.K = (int)a.size(1);
  args.N = (int)b.size(0);
  TORCH_CHECK(b.size(1) == args.K, "gemm_peer: K mismatch");
  args.k_splits = 1;
  if (bias.has_value()) {
    need(*bias, at::kBFloat16, "bias");
    TORCH_CHECK(bias->is_contiguous() && bias->numel() == args.N, "gemm_peer: bias [N]");
    args.bias = cbf(*bias);
  }
  args.vec_ok = (ld % 8 == 0 && col_off % 8 == 0 && slot_stride % 8 == 0) ? 1 : 0;
  args.err = err.data_ptr<int>();
  args.peer.n_peers = (int)peers.size();
  for (size_t i = 0; i < peers.size(); ++i) args.peer.peer[i] = reinterpret_cast<void*>(peers[i]);
  args.peer.mode = (int)mode;
  args.peer.slot = (int)slot;
  args.peer.row_chunk = (int)row_chunk;
  args.peer.slot_stride = slot_stride;
  args.peer.ld = ld;
  args.peer.col_off = col_off;
  rf::gemm_bf16(op, args, rf::kEpiPeer, (int)bn, 0, cur());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Row-parallel product fused with its all-reduce through NVSwitch multicast (kEpiNvlsAR): out_part is this
// rank's symmetric partial buffer (unicast view), mc_part / mc_out the multicast addresses of the partial and
// output buffers.
void gemm_nvls_ar_b(Tensor a, Tensor b, c10::optional<Tensor> residual, Tensor out_part, int64_t mc_part,
                    int64_t mc_out, int64_t flags_local, std::vector<int64_t> flag_peers, int64_t rank, int64_t epoch,
                    Tensor counters, int64_t max_mb, int64_t bn, int64_t max_ctas, Tensor err, bool comm_off,
                    int64_t comm_ctas) {
  need(a, at::kBFloat16, "a");
  need(b, at::kBFloat16, "b");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && out_part.stride(1) == 1, "gemm_nvls_ar: unit inner stride");
  TORCH_CHECK(flag_peers.size() >= 1 && flag_peers.size() <= rf::kMaxPeers, "gemm_nvls_ar: 1..8 ranks");
  TORCH_CHECK(counters.scalar_type() == at::kInt && counters.numel() >= max_mb + 1, "gemm_nvls_ar: counters");
  c10::cuda::CUDAGuard g(a.device());
  rf::GemmOperands op{a.data_ptr(), a.stride(0), false, b.data_ptr(), b.stride(0), false};
  rf::GemmArgs args{};
  args.M = (int)a.size(0);
  args.K = (int)a.size(1);
  args.N = (int)b.size(0);
  TORCH_CHECK(b.size(1) == args.K && out_part.size(0) == args.M && out_part.size(1) == args.N, "gemm_nvls_ar: shapes");
  TORCH_CHECK(args.N % 8 == 0 && out_part.stride(0) % 8 == 0, "gemm_nvls_ar: N and the row pitch must be multiples of 8");
  TORCH_CHECK((args.M + 127) / 128 <= max_mb, "gemm_nvls_ar: more row blocks than the flag array holds");
  args.k_splits = 1;
  args.out = out_part.data_ptr();
  args.ldo = out_part.stride(0);
  if (residual.has_value()) {
    need(*residual, at::kBFloat16, "residual");
    TORCH_CHECK(residual->stride(1) == 1 && residual->size(0) == args.M && residual->size(1) == args.N,
                "gemm_nvls_ar: residual [M, N]");
    args.residual = cbf(*residual);
    args.ldr = residual->stride(0);
  }
  args.vec_ok = (args.ldo % 8 == 0 && (!residual.has_value() || args.ldr % 8 == 0)) ? 1 : 0;
  args.err = err.data_ptr<int>();
  rf::NvlsGemmArgs& nv = args.nvls;
  nv.mc_part = reinterpret_cast<const void*>(mc_part);
  nv.mc_out = reinterpret_cast<void*>(mc_out);
  nv.flags = reinterpret_cast<int*>(flags_local);
  for (size_t i = 0; i < flag_peers.size(); ++i) nv.peer_flags[i] = reinterpret_cast<int*>(flag_peers[i]);
  nv.world = (int)flag_peers.size();
  nv.rank = (int)rank;
  nv.epoch = (int)epoch;
  nv.rb_count = counters.data_ptr<int>();
  nv.done_count = counters.data_ptr<int>() + max_mb;
  nv.max_mb = (int)max_mb;
  nv.comm_off = comm_off ? 1 : 0;
  nv.comm_ctas = (int)comm_ctas;
  rf::gemm_bf16(op, args, rf::kEpiNvlsAR, (int)bn, (int)max_ctas, cur());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// Column-sharded product fused with its all-gather through NVSwitch multicast (kEpiNvlsAG): this rank's columns
// of x = a b^T + bias land in every rank's copy of the full [M, d] buffer (mc_full: its multicast address).
void gemm_nvls_ag_b(Tensor a, Tensor b, c10::optional<Tensor> bias, int64_t mc_full, int64_t d, int64_t col_off,
                    int64_t flags_local, std::vector<int64_t> flag_peers, int64_t rank, int64_t epoch, Tensor counters,
                    int64_t bn, Tensor err) {
  need(a, at::kBFloat16, "a");
  need(b, at::kBFloat16, "b");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1, "gemm_nvls_ag: unit inner stride");
  TORCH_CHECK(flag_peers.size() >= 1 && flag_peers.size() <= rf::kMaxPeers, "gemm_nvls_ag: 1..8 ranks");
  c10::cuda::CUDAGuard g(a.device());
  rf::GemmOperands op{a.data_ptr(), a.stride(0), false, b.data_ptr(), b.stride(0), false};
  rf::GemmArgs args{};
  args.M = (int)a.size(0);
  args.K = (int)a.size(1);
  args.N = (int)b.size(0);
  TORCH_CHECK(b.size(1) == args.K, "gemm_nvls_ag: K mismatch");
  TORCH_CHECK(args.N % 64 == 0 && d % 8 == 0 && col_off % 8 == 0 && col_off + args.N <= d,
              "gemm_nvls_ag: column slice must be whole 64-column chunks inside d, 16-byte aligned");
  args.k_splits = 1;
  args.out = reinterpret_cast<void*>(mc_full + col_off * 2);
  args.ldo = d;
  if (bias.has_value()) {
    need(*bias, at::kBFloat16, "bias");
    TORCH_CHECK(bias->is_contiguous() && bias->numel() == args.N, "gemm_nvls_ag: bias [N]");
    args.bias = cbf(*bias);
  }
  args.vec_ok = 1;
  args.err = err.data_ptr<int>();
  rf::NvlsGemmArgs& nv = args.nvls;
  nv.flags = reinterpret_cast<int*>(flags_local);
  for (size_t i = 0; i < flag_peers.size(); ++i) nv.peer_flags[i] = reinterpret_cast<int*>(flag_peers[i]);
  nv.world = (int)flag_peers.size();
  nv.rank = (int)rank;
  nv.epoch = (int)epoch;
  TORCH_CHECK(counters.scalar_type() == at::kInt && counters.numel() >= 1, "gemm_nvls_ag: counters");
  nv.done_count = counters.data_ptr<int>();
  nv.max_mb = 0;
  rf::gemm_bf16(op, args, rf::kEpiNvlsAG, (int)bn, 0, cur());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

}  // namespace

void router_topk_b(Tensor logits, int64_t E, int64_t k, Tensor idx, Tensor wts, bool norm) {
  need(logits, at::kFloat, "logits");
  need(idx, at::kInt, "idx");
  need(wts, at::kFloat, "wts");
  TORCH_CHECK(E <= 1024 && k <= 16 && logits.stride(1) == 1, "router_topk: E <= 1024, k <= 16");
  rf::router_topk(logits.data_ptr<float>(), logits.stride(0), (int)logits.size(0), (int)E, (int)k,
                  idx.data_ptr<int>(), wts.data_ptr<float>(), norm ? 1 : 0, cur());
}

void moe_align_b(Tensor idx, int64_t e0, int64_t E, Tensor counts, Tensor rank, Tensor seg_start, Tensor tile_start, Tensor pos,
                 Tensor x, Tensor xp) {
  need(idx, at::kInt, "idx");
  need(x, at::kBFloat16, "x");
  need(xp, at::kBFloat16, "xp");
  TORCH_CHECK(E <= 4096 && x.size(1) % 8 == 0 && x.stride(1) == 1, "moe_align: E <= 4096, d % 8");
  const int n = (int)idx.size(0), k = (int)idx.size(1);
  rf::moe_align(idx.data_ptr<int>(), n, k, (int)e0, (int)E, counts.data_ptr<int>(), rank.data_ptr<int>(),
                seg_start.data_ptr<int>(), tile_start.data_ptr<int>(), pos.data_ptr<int>(), cbf(x), x.stride(0), bf(xp),
                (int)x.size(1), cur());
}

void grouped_gemm_b(Tensor xp, Tensor w, Tensor seg_start, Tensor tile_start, Tensor out, bool swiglu, Tensor err) {
  need(xp, at::kBFloat16, "xp");
  need(w, at::kBFloat16, "w");
  need(out, at::kBFloat16, "out");
  TORCH_CHECK(w.dim() == 3 && w.is_contiguous() && xp.is_contiguous(), "grouped_gemm: w [E, N, K] contiguous");
  TORCH_CHECK(w.size(2) == xp.size(1), "grouped_gemm: K mismatch");
  c10::cuda::CUDAGuard g(xp.device());
  rf::grouped_gemm(cbf(xp), xp.size(0), cbf(w), (int)w.size(0), (int)w.size(1), (int)w.size(2),
                   seg_start.data_ptr<int>(), tile_start.data_ptr<int>(), bf(out), out.stride(0), swiglu ? 1 : 0,
                   err.data_ptr<int>(), cur());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void moe_combine_b(c10::optional<Tensor> h_opt, Tensor y, Tensor pos, Tensor w, c10::optional<Tensor> ys,
                   c10::optional<Tensor> gate_logit, Tensor out) {
  need(out, at::kBFloat16, "out");
  const __nv_bfloat16* hp = h_opt.has_value() ? cbf(*h_opt) : nullptr;
  const long ldh = h_opt.has_value() ? h_opt->stride(0) : 0;
  const Tensor& h = out;
  need(y, at::kBFloat16, "y");
  need(out, at::kBFloat16, "out");
  const int n = (int)h.size(0), k = (int)pos.size(1), d = (int)h.size(1);
  const __nv_bfloat16* ysp = ys.has_value() ? cbf(*ys) : nullptr;
  const float* gl = gate_logit.has_value() ? gate_logit->data_ptr<float>() : nullptr;
  const long ldg = gate_logit.has_value() ? gate_logit->stride(0) : 0;
  rf::moe_combine(hp, ldh, cbf(y), pos.data_ptr<int>(), w.data_ptr<float>(), n, k, ysp, gl, ldg, bf(out), d,
                  cur());
}

void score_rows_b(Tensor logits, c10::optional<Tensor> ref, c10::optional<Tensor> targets, Tensor logprob, Tensor lse,
                  Tensor argmax, Tensor ref_argmax, Tensor kl) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == torch::kFloat32 && logits.dim() == 2 && logits.stride(1) == 1,
              "score_rows: fp32 [rows, V] logits with unit column stride");
  const int rows = (int)logits.size(0), V = (int)logits.size(1);
  rf::ScoreArgs a{};
  a.logits = logits.data_ptr<float>();
  a.ld = logits.stride(0);
  a.rows = rows;
  a.V = V;
  if (ref.has_value()) {
    TORCH_CHECK(ref->scalar_type() == torch::kFloat32 && ref->size(0) == rows && ref->size(1) == V && ref->stride(1) == 1,
                "score_rows: ref must match logits");
    a.ref = ref->data_ptr<float>();
    a.ld_ref = ref->stride(0);
    a.kl = kl.data_ptr<double>();
    a.ref_argmax = ref_argmax.data_ptr<int>();
  }
  if (targets.has_value()) {
    TORCH_CHECK(targets->scalar_type() == torch::kInt64 && targets->numel() == rows, "score_rows: int64 targets [rows]");
    a.targets = targets->data_ptr<int64_t>();
    a.logprob = logprob.data_ptr<double>();
  }
  a.lse = lse.data_ptr<double>();
  a.argmax = argmax.data_ptr<int>();
  rf::score_rows(a, at::cuda::getCurrentCUDAStream());
}

rf::NvlsFlags nvls_flags_of(int64_t local, const std::vector<int64_t>& peers, int64_t rank) {
  rf::NvlsFlags f{};
  TORCH_CHECK(peers.size() >= 1 && peers.size() <= rf::kMaxRanksNvls, "nvls: 1..8 ranks");
  f.local = reinterpret_cast<int*>(local);
  f.world = (int)peers.size();
  f.rank = (int)rank;
  for (size_t i = 0; i < peers.size(); ++i) f.peer[i] = reinterpret_cast<int*>(peers[i]);
  return f;
}

void nvls_allreduce_b(int64_t mc_in, int64_t mc_out, int64_t out_local, c10::optional<Tensor> dst, int64_t rows,
                      int64_t d, int64_t row0, int64_t row1, int64_t flags_local, std::vector<int64_t> flag_peers,
                      int64_t rank, int64_t slot_in, int64_t slot_out, int64_t epoch, int64_t counter, Tensor err,
                      int64_t max_ctas, bool acc32) {
  TORCH_CHECK(d % 8 == 0, "nvls_allreduce: d must be a multiple of 8");
  rf::NvlsAllReduceArgs a{};
  a.mc_in = reinterpret_cast<const void*>(mc_in);
  a.mc_out = reinterpret_cast<void*>(mc_out);
  a.out_local = reinterpret_cast<const __nv_bfloat16*>(out_local);
  if (dst.has_value()) {
    TORCH_CHECK(dst->is_contiguous() && dst->scalar_type() == torch::kBFloat16 && dst->numel() == rows * d,
                "nvls_allreduce: dst must be a contiguous bf16 [rows, d] tensor");
    a.dst = reinterpret_cast<__nv_bfloat16*>(dst->data_ptr());
  }
  a.rows = (int)rows;
  a.d = (int)d;
  a.row0 = (int)row0;
  a.row1 = (int)row1;
  a.f = nvls_flags_of(flags_local, flag_peers, rank);
  a.slot_in = (int)slot_in;
  a.slot_out = (int)slot_out;
  a.epoch = (int)epoch;
  a.counter = reinterpret_cast<int*>(counter);
  a.err = err.data_ptr<int>();
  a.max_ctas = (int)max_ctas;
  a.acc32 = acc32 ? 1 : 0;
  rf::nvls_allreduce(a, cur());
}

void nvls_allreduce_f64_b(int64_t mc_in, int64_t mc_out, int64_t n, int64_t flags_local,
                          std::vector<int64_t> flag_peers, int64_t rank, int64_t slot_in, int64_t slot_out,
                          int64_t epoch, int64_t counter, Tensor err) {
  rf::NvlsAllReduceF64Args a{};
  a.mc_in = reinterpret_cast<const void*>(mc_in);
  a.mc_out = reinterpret_cast<void*>(mc_out);
  a.n = n;
  a.f = nvls_flags_of(flags_local, flag_peers, rank);
  a.slot_in = (int)slot_in;
  a.slot_out = (int)slot_out;
  a.epoch = (int)epoch;
  a.counter = reinterpret_cast<int*>(counter);
  a.err = err.data_ptr<int>();
  rf::nvls_allreduce_f64(a, cur());
}

void nvls_allgather_b(Tensor src, int64_t mc_out, int64_t d, int64_t col_off, int64_t flags_local,
                      std::vector<int64_t> flag_peers, int64_t rank, int64_t slot, int64_t epoch, int64_t counter,
                      Tensor err) {
  TORCH_CHECK(src.is_cuda() && src.scalar_type() == torch::kBFloat16 && src.dim() == 2 && src.stride(1) == 1 &&
                  src.size(1) % 8 == 0 && src.stride(0) % 8 == 0 && col_off % 8 == 0 && d % 8 == 0,
              "nvls_allgather: bf16 [rows, cols] slice, 16-byte aligned rows and offsets");
  rf::NvlsAllGatherArgs a{};
  a.src = reinterpret_cast<const __nv_bfloat16*>(src.data_ptr());
  a.ld_src = src.stride(0);
  a.mc_out = reinterpret_cast<void*>(mc_out);
  a.rows = (int)src.size(0);
  a.cols = (int)src.size(1);
  a.d = (int)d;
  a.col_off = (int)col_off;
  a.f = nvls_flags_of(flags_local, flag_peers, rank);
  a.slot = (int)slot;
  a.epoch = (int)epoch;
  a.counter = reinterpret_cast<int*>(counter);
  a.err = err.data_ptr<int>();
  rf::nvls_allgather(a, cur());
}

void nvls_barrier_b(int64_t flags_local, std::vector<int64_t> flag_peers, int64_t rank, int64_t slot, int64_t epoch,
                    Tensor err) {
  rf::nvls_barrier(nvls_flags_of(flags_local, flag_peers, rank), (int)slot, (int)epoch, err.data_ptr<int>(), cur());
}

void row_cosine_b(Tensor a, Tensor b, Tensor out, double eps) {
  need(a, at::kBFloat16, "a");
  need(b, at::kBFloat16, "b");
  need(out, at::kFloat, "out");
  TORCH_CHECK(a.dim() == 2 && b.sizes() == a.sizes() && a.stride(1) == 1 && b.stride(1) == 1 &&
                  out.numel() == a.size(0),
              "row_cosine: a, b [rows, d] with unit column stride, out [rows]");
  rf::row_cosine(cbf(a), a.stride(0), cbf(b), b.stride(0), a.size(0), (int)a.size(1), (float)eps,
                 out.data_ptr<float>(), cur());
}

void window_mass_b(Tensor q, Tensor k, Tensor qpos, double scale, Tensor mass, Tensor part_m, Tensor part_l, Tensor qm,
                   Tensor ql) {
  need(q, at::kBFloat16, "q");
  need(k, at::kBFloat16, "k");
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && q.size(2) == k.size(2) && q.stride(2) == 1 && k.stride(2) == 1,
              "window_mass: q [hq, w, hd], k [hkv, n, hd]");
  const int hd = (int)q.size(2);
  TORCH_CHECK(hd % 16 == 0 && hd <= 256 && q.stride(1) % 8 == 0 && q.stride(0) % 8 == 0 && k.stride(1) % 8 == 0 &&
                  k.stride(0) % 8 == 0 && q.size(0) % k.size(0) == 0,
              "window_mass: head_dim a multiple of 16 (<= 256), 16-byte aligned rows, GQA");
  TORCH_CHECK(qpos.scalar_type() == at::kInt && qpos.numel() == q.size(1), "window_mass: int32 qpos [w]");
  TORCH_CHECK(mass.scalar_type() == at::kDouble && mass.numel() >= k.size(1), "window_mass: fp64 mass [n]");
  rf::WindowMassArgs a{};
  a.q = cbf(q);
  a.q_head_stride = q.stride(0);
  a.q_row_stride = q.stride(1);
  a.k = cbf(k);
  a.k_head_stride = k.stride(0);
  a.k_row_stride = k.stride(1);
  a.qpos = qpos.data_ptr<int>();
  a.hq = (int)q.size(0);
  a.hkv = (int)k.size(0);
  a.w = (int)q.size(1);
  a.n = (int)k.size(1);
  a.hd = hd;
  a.scale = (float)scale;
  const long nblk = (a.n + 63) / 64;
  TORCH_CHECK(part_m.numel() >= (long)a.hq * a.w * nblk && part_l.numel() >= (long)a.hq * a.w * nblk &&
                  qm.numel() >= (long)a.hq * a.w && ql.numel() >= (long)a.hq * a.w,
              "window_mass: scratch sizes");
  a.part_m = part_m.data_ptr<float>();
  a.part_l = part_l.data_ptr<float>();
  a.qm = qm.data_ptr<float>();
  a.ql = ql.data_ptr<float>();
  a.mass = mass.data_ptr<double>();
  rf::window_mass(a, cur());
}

void cholesky_solve_b(Tensor a, Tensor b, double shift, Tensor err) {
  need(a, at::kDouble, "a");
  need(b, at::kDouble, "b");
  TORCH_CHECK(a.dim() == 2 && a.size(0) == a.size(1) && a.stride(1) == 1 && b.stride(1) == 1 &&
                  b.size(0) == a.size(0), "cholesky_solve: a [n, n], b [n, R]");
  c10::cuda::CUDAGuard g(a.device());
  rf::cholesky_solve(a.data_ptr<double>(), (int)a.size(0), a.stride(0), shift, b.data_ptr<double>(), b.stride(0),
                     (int)b.size(1), err.data_ptr<int>(), cur());
}

void register_comm(pybind11::module_& m) {
  m.def("cholesky_solve", &cholesky_solve_b);
  m.def("score_rows", &score_rows_b);
  m.def("row_cosine", &row_cosine_b);
  m.def("window_mass", &window_mass_b);
  m.def("nvls_allreduce", &nvls_allreduce_b);
  m.def("nvls_allgather", &nvls_allgather_b);
  m.def("nvls_allreduce_f64", &nvls_allreduce_f64_b);
  m.def("nvls_barrier", &nvls_barrier_b);
  m.def("router_topk", &router_topk_b);
  m.def("moe_align", &moe_align_b);
  m.def("grouped_gemm", &grouped_gemm_b);
  m.def("moe_combine", &moe_combine_b);
  m.def("ipc_malloc", &ipc_malloc_b);
  m.def("ipc_free", &ipc_free_b);
  m.def("ipc_handle", &ipc_handle_b);
  m.def("ipc_open", &ipc_open_b);
  m.def("ipc_close", &ipc_close_b);
  m.def("tensor_at", &tensor_at);
  m.def("comm_signal", &comm_signal_b);
  m.def("comm_wait", &comm_wait_b, pybind11::arg("flags"), pybind11::arg("first"), pybind11::arg("n"),
        pybind11::arg("value"), pybind11::arg("err"), pybind11::arg("limit_ns") = 0);
  m.def("comm_reduce_rows", &comm_reduce_rows_b);
  m.def("comm_gather_rows", &comm_gather_rows_b);
  m.def("gemm_peer", &gemm_peer_b);
  m.def("gemm_nvls_ar", &gemm_nvls_ar_b);
  m.def("gemm_nvls_ag", &gemm_nvls_ag_b);
}
