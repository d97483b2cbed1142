// ta_api.cu -- host side of the C ABI (include/turboadam_b200.h): argument
// validation, per-tensor constant derivation (exactly as torch rounds the
// Python scalars), workspace carving, multi-tensor launch lists and the
// fixed kernel sequence of one optimizer step.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/turboadam_b200.h"
#include "ta_codec.cuh"
#include "ta_kernels.cuh"

using namespace ta;

namespace {

thread_local std::string g_err;

ta_status fail(ta_status s, const std::string& m) {
  g_err = m;
  return s;
}

#define TA_CU(x)                                                                  \
  do {                                                                            \
    cudaError_t e_ = (x);                                                         \
    if (e_ != cudaSuccess)                                                        \
      return fail(TA_ERR_CUDA, std::string(#x) + ": " + cudaGetErrorString(e_));  \
  } while (0)

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }
inline bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// Python int(pct * n) (trunc toward zero of an IEEE double product),
// costate.py:116-117.
void threshold_ranks(int64_t B, double null_pct, double amp_pct, int64_t* lo, int64_t* hi) {
  int64_t a = (int64_t)(null_pct * (double)B) - 1;
  int64_t b = (int64_t)(amp_pct * (double)B);
  *lo = a < 0 ? 0 : a;
  *hi = b > B - 1 ? B - 1 : b;
}

// ---- workspace layout ---------------------------------------------------
constexpr int kMaxLists = 40;

struct CsSlot {
  size_t part, ratios, hist, sel, alpha, chunk, efd;
};

struct Layout {
  size_t status = 0;
  size_t table = 0;
  size_t lists = 0;
  size_t list_stride = 0;
  size_t sel_block = 0;    // the select state of every CoState tensor, contiguous
  size_t sel_bytes = 0;    //   (cleared at the start of each step)
  std::vector<CsSlot> cs;  // per CoState tensor
  size_t total = 0;
};

// cs_bpad: padded blocks of each CoState tensor, negative for one with error
// feedback (which also gets a delta buffer of that many blocks).
Layout layout_for(int nT, const std::vector<int64_t>& cs_bpad) {
  Layout L;
  size_t off = 0;
  L.status = off;
  off += 256;
  L.table = off;
  off = al256(off + (size_t)nT * sizeof(DevTensor));
  L.lists = off;
  L.list_stride = al256((size_t)(nT + 1) * sizeof(int64_t) + (size_t)nT * sizeof(int32_t));
  off += L.list_stride * kMaxLists;
  L.sel_block = off;
  L.sel_bytes = al256(cs_bpad.size() * 16 * 4);
  off += L.sel_bytes;
  size_t ci = 0;
  for (int64_t sbp : cs_bpad) {
    const int64_t bp = sbp < 0 ? -sbp : sbp;
    CsSlot s;
    s.sel = L.sel_block + 16 * 4 * ci++;
    s.part = off;
    off = al256(off + (size_t)bp * 2 * 4);
    s.ratios = off;
    off = al256(off + (size_t)bp * 4);
    s.hist = off;
    off = al256(off + (size_t)3 * 2 * HBINS * 4);
    s.alpha = off;
    off = al256(off + 4 * 4);
    s.chunk = off;
    off = al256(off + (size_t)2 * cdiv(bp / TB, FIN_THREADS) * 8);
    s.efd = 0;
    if (sbp < 0) {
      s.efd = off;
      off = al256(off + (size_t)bp * BS * 4);
    }
    L.cs.push_back(s);
  }
  L.total = off;
  return L;
}

bool is_costate(const ta_tensor& t) { return (t.flags & TA_M_COSTATE) != 0; }

std::vector<int64_t> cs_bpads(const ta_tensor* ts, int n) {
  std::vector<int64_t> v;
  for (int i = 0; i < n; ++i)
    if (ts[i].numel > 0 && is_costate(ts[i])) {
      const int64_t bp = cdiv(cdiv(ts[i].numel, BS), TB) * TB;
      v.push_back((ts[i].flags & TA_M_EF) ? -bp : bp);
    }
  return v;
}

bool is_spanning(const ta_tensor& t) {
  return t.numel > 0 && is_costate(t) && (t.flags & TA_M_SPANNING) != 0;
}

// Exchange slot sizes of one split tensor (elements).
inline int64_t xchunk_elems(int64_t global_blocks) {
  return 2 * cdiv(cdiv(global_blocks, TB), FIN_THREADS);
}
constexpr int64_t kXHistElems = 2 * HBINS;

// ---- kernel registry (one-time attribute setup, occupancy) --------------
template <typename K>
int setup_kernel(K kern, size_t smem, int threads) {
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  int occ = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, threads, smem);
  return occ > 0 ? occ : 1;
}

struct LaunchList {
  std::vector<int64_t> beg;  // tile (or chunk) prefix, size n+1
  std::vector<int32_t> idx;
};

template <int MK, int VK, int PT, bool UNI, bool TABLE>
ta_status launch_p1(const KParams& kp, cudaStream_t s) {
  constexpr size_t smem = p1_smem_bytes<MK, VK, PT, UNI>();
  static std::once_flag once;
  static int occ = 1;
  std::call_once(once, [] { occ = setup_kernel(k_pass1<MK, VK, PT, UNI, TABLE>, smem, NTHR); });
  int64_t grid = std::min<int64_t>(kp.total, (int64_t)sm_count() * occ);
  if (grid <= 0) return TA_OK;
  k_pass1<MK, VK, PT, UNI, TABLE><<<(unsigned)grid, NTHR, smem, s>>>(kp);
  TA_CU(cudaGetLastError());
  return TA_OK;
}

template <int MK, int VK, int PT>
ta_status launch_p1_u(bool uni, bool table, const KParams& kp, cudaStream_t s) {
  if (VK != VK_ONEQ)  // uniforms and the exp table only matter for 1Q
    return launch_p1<MK, VK, PT, false, false>(kp, s);
  if (uni)
    return table ? launch_p1<MK, VK, PT, true, true>(kp, s)
                 : launch_p1<MK, VK, PT, true, false>(kp, s);
  return table ? launch_p1<MK, VK, PT, false, true>(kp, s)
               : launch_p1<MK, VK, PT, false, false>(kp, s);
}

ta_status dispatch_p1(int mk, int vk, int pt, bool uni, bool table, const KParams& kp,
                      cudaStream_t s) {
#define TA_P1(M, V)                                                               \
  if (mk == M && vk == V)                                                         \
    return pt ? launch_p1_u<M, V, 1>(uni, table, kp, s)                           \
              : launch_p1_u<M, V, 0>(uni, table, kp, s);
  TA_P1(MK_COSTATE, VK_ONEQ)
  TA_P1(MK_COSTATE, VK_FP32)
  TA_P1(MK_COSTATE, VK_NONE)
  TA_P1(MK_FP32, VK_ONEQ)
  TA_P1(MK_FP32, VK_FP32)
  TA_P1(MK_NONE, VK_ONEQ)
#undef TA_P1
  return fail(TA_ERR_UNSUPPORTED, "moment combination not built");
}

template <int PT>
ta_status launch_p2(const KParams& kp, cudaStream_t s) {
  constexpr size_t smem = p2_smem_bytes<PT>();
  static std::once_flag once;
  static int occ = 1;
  std::call_once(once, [] { occ = setup_kernel(k_pass2<PT>, smem, NTHR); });
  int64_t grid = std::min<int64_t>(kp.total, (int64_t)sm_count() * occ);
  if (grid <= 0) return TA_OK;
  k_pass2<PT><<<(unsigned)grid, NTHR, smem, s>>>(kp);
  TA_CU(cudaGetLastError());
  return TA_OK;
}

int mk_of(const ta_tensor& t) {
  if (t.flags & TA_M_COSTATE) return MK_COSTATE;
  return t.exp_avg_dev ? MK_FP32 : MK_NONE;
}
int vk_of(const ta_tensor& t) {
  if (t.flags & TA_V_ONEQ) return VK_ONEQ;
  return t.exp_avg_sq_dev ? VK_FP32 : VK_NONE;
}

ta_status validate(const ta_tensor& t, int i, int n_groups, const ta_group* groups) {
  auto bad = [&](const char* what) {
    return fail(TA_ERR_INVALID, "tensor " + std::to_string(i) + ": " + what);
  };
  if (t.numel < 0) return bad("negative numel");
  if (t.numel == 0) return TA_OK;
  if (t.dtype != TA_F32 && t.dtype != TA_BF16) return bad("dtype must be TA_F32 or TA_BF16");
  if (t.group < 0 || t.group >= n_groups) return bad("group index out of range");
  const ta_group& g = groups[t.group];
  if (g.block_size != BS)
    return fail(TA_ERR_UNSUPPORTED, "tensor " + std::to_string(i) + ": block_size " +
                                        std::to_string(g.block_size) + " (only 128 is built)");
  if ((t.flags & TA_V_ONEQ) && !(g.v_bits == 2 || g.v_bits == 3 || g.v_bits == 4 ||
                                 g.v_bits == 6 || g.v_bits == 8))
    return bad("v_bits must be one of {2, 3, 4, 6, 8}");
  if (t.step == 0) return bad("step must be >= 1 (count after increment)");
  const bool param = !(t.flags & TA_NO_PARAM);
  if (!t.grad_dev) return bad("null grad");
  if (param && !t.param_dev) return bad("null param");
  const int mk = mk_of(t), vk = vk_of(t);
  if (param && (mk == MK_NONE || vk == VK_NONE))
    return bad("parameter update needs both moments (set exp_avg / exp_avg_sq or flags)");
  if (mk == MK_COSTATE && (!t.m_labels_dev || !t.m_signs_dev || !t.m_norms_dev ||
                           !t.m_amp_dev || !t.m_alpha_dev))
    return bad("CoState state pointer missing");
  if (vk == VK_ONEQ && (!t.v_idx_dev || !t.v_hdr_dev)) return bad("1Q state pointer missing");
  if (t.block_offset < 0 || t.global_blocks < 0) return bad("negative shard offset / size");
  const int64_t nb_local = cdiv(t.numel, BS);
  if (t.global_blocks && t.block_offset + nb_local > t.global_blocks)
    return bad("shard extends past global_blocks");
  if ((t.flags & TA_M_EF) && (mk != MK_COSTATE || !t.m_ef_dev))
    return bad("TA_M_EF needs a CoState first moment and m_ef_dev");
  if (t.flags & TA_M_SPANNING) {
    if (mk != MK_COSTATE) return bad("TA_M_SPANNING needs a CoState first moment");
    if (t.block_offset % TA_SHARD_ALIGN_BLOCKS)
      return bad("a spanning shard must start at a multiple of TA_SHARD_ALIGN_BLOCKS blocks");
    if (t.block_offset + nb_local < t.global_blocks && t.numel % BS)
      return bad("only the last shard of a tensor may end in a partial block");
  }
  const void* al[] = {t.param_dev, t.grad_dev, t.v_idx_dev, t.v_hdr_dev, t.exp_avg_sq_dev,
                      t.m_labels_dev, t.m_signs_dev, t.m_norms_dev, t.m_amp_dev, t.exp_avg_dev,
                      t.sr_uniforms_dev, t.m_ef_dev};
  for (const void* p : al)
    if (p && !aligned16(p))
      return fail(TA_ERR_ALIGN, "tensor " + std::to_string(i) + ": pointer not 16-byte aligned");
  return TA_OK;
}

DevTensor make_dev(const ta_tensor& t, const ta_group& g, uint64_t seed) {
  DevTensor D;
  memset(&D, 0, sizeof(D));
  D.p = t.param_dev;
  D.g = t.grad_dev;
  D.v_idx = t.v_idx_dev;
  D.v_hdr = t.v_hdr_dev;
  D.eas = t.exp_avg_sq_dev;
  D.lab = t.m_labels_dev;
  D.sgn = t.m_signs_dev;
  D.nrm = t.m_norms_dev;
  D.amp = t.m_amp_dev;
  D.alpha_state = t.m_alpha_dev;
  D.ea = t.exp_avg_dev;
  D.uni = t.sr_uniforms_dev;
  D.alpha_inj = t.alpha_inject_dev;
  D.m_out = t.m_out_dev;
  D.v_out = t.v_out_dev;
  D.ef = t.m_ef_dev;
  D.n = t.numel;
  D.nblk = cdiv(t.numel, BS);
  D.bpad = cdiv(D.nblk, TB) * TB;
  const int64_t gblocks = t.global_blocks ? t.global_blocks : D.nblk;
  threshold_ranks(gblocks, g.null_pct, g.amp_pct, &D.k_lo, &D.k_hi);
  D.boff = t.block_offset;
  D.cglob = cdiv(cdiv(gblocks, TB), FIN_THREADS);
  D.coff = t.block_offset / (TB * FIN_THREADS);
  // fp32 values of the Python scalars exactly as torch rounds them
  D.b1 = (float)g.beta1;
  D.omb1 = (float)(1.0 - g.beta1);
  D.b2 = (float)g.beta2;
  D.omb2 = (float)(1.0 - g.beta2);
  D.wdf = (float)(1.0 - g.lr * g.weight_decay);
  D.nlr = (float)(-g.lr);
  D.eps = (float)g.eps;
  D.bc1 = g.bc1;
  D.bc2 = g.bc2;
  D.rbc2 = 1.0f / g.bc2;
  D.nbits = g.v_bits;
  D.nbf = (float)(1 << g.v_bits);
  D.sqbs = (float)std::sqrt((double)g.block_size);
  D.rsqbs = 1.0f / D.sqbs;
  uint32_t f = 0;
  if (t.flags & TA_M_COSTATE) f |= DF_M_COSTATE;
  if (t.flags & TA_V_ONEQ) f |= DF_V_ONEQ;
  if (t.flags & TA_M_HAS_STATE) f |= DF_M_HAS_STATE;
  if (t.flags & TA_NO_PARAM) f |= DF_NO_PARAM;
  if (g.weight_decay != 0.0) f |= DF_WD;
  if (t.sr_uniforms_dev) f |= DF_UNI;
  if (t.alpha_inject_dev) f |= DF_ALPHA_INJ;
  if (t.m_out_dev) f |= DF_M_OUT;
  if (t.v_out_dev) f |= DF_V_OUT;
  if (t.dtype == TA_BF16) f |= DF_BF16;
  if (t.flags & TA_M_SPANNING) f |= DF_SPAN;
  if (t.flags & TA_EXACT_PARAM) f |= DF_EXACT_P;
  if (t.flags & TA_M_EF) f |= DF_EF;
  if ((t.flags & TA_M_EF) && (t.flags & TA_M_EF_STATE)) f |= DF_EF_STATE;
  D.flags = f;
  D.tid = t.tensor_id;
  D.step = t.step;
  D.seed_lo = (uint32_t)seed;
  D.seed_hi = (uint32_t)(seed >> 32);
  D.sel_chunks = (int32_t)cdiv(D.bpad, SEL_CHUNK);
  D.alpha_chunks = (int32_t)cdiv(D.bpad / TB, FIN_THREADS);
  D.one = 1.0f;
  D.group = t.group;
  D.ginv = 1.0f;
  D.wdd = g.weight_decay;
  return D;
}

// Runs the fixed kernel sequence for an already validated tensor list.
// ev (optional, 5 entries, may be null individually): cudaEvent_t recorded on
// `st` before pass 1, after pass 1, after alpha, after pass 2, after labels.
struct P1Key { int mk, vk, pt; bool uni, table; };

// Error-feedback residual update of the EF tensors (after the labels).
ta_status launch_ef(const KParams& efk, cudaStream_t st) {
  if (!efk.total) return TA_OK;
  const int64_t grid = std::min<int64_t>(efk.total, (int64_t)sm_count() * 8);
  k_ef<<<(unsigned)grid, 256, 0, st>>>(efk);
  TA_CU(cudaGetLastError());
  return TA_OK;
}

// One phase of a sharded step (TA_PHASE_*), after the descriptors are uploaded.
ta_status run_phase(int phase, const std::vector<std::pair<P1Key, LaunchList>>& p1,
                    const std::vector<KParams>& p1k, const KParams* p2k, const SelParams& ap,
                    int64_t achunks, const SelParams& sp, int64_t nchunks, const SelParams& xap,
                    unsigned xa_chunks, const SelParams& xsp, unsigned xsel_chunks,
                    const SelParams& xp, unsigned nx, const KParams& efk, uint8_t* exch,
                    size_t chunk_bytes, size_t hist_bytes, cudaStream_t st) {
  uint8_t* xh = exch + chunk_bytes;
  switch (phase) {
    case TA_PHASE_PASS1:
      for (size_t i = 0; i < p1.size(); ++i) {
        const P1Key& k = p1[i].first;
        ta_status r = dispatch_p1(k.mk, k.vk, k.pt, k.uni, k.table, p1k[i], st);
        if (r != TA_OK) return r;
      }
      if (achunks) k_alpha<<<(unsigned)achunks, FIN_THREADS, 0, st>>>(ap);
      // every rank clears its regions (also one without split tensors: its
      // zeros take part in the sum)
      if (exch && chunk_bytes) TA_CU(cudaMemsetAsync(exch, 0, chunk_bytes, st));
      if (nx) k_alpha_part<<<xa_chunks, FIN_THREADS, 0, st>>>(xap);
      break;
    case TA_PHASE_PASS2:
      if (nx) k_alpha_fin<<<nx, FIN_THREADS, 0, st>>>(xp);
      for (int pt = 0; pt < 2; ++pt) {
        if (!p2k[pt].total) continue;
        ta_status r = pt ? launch_p2<1>(p2k[pt], st) : launch_p2<0>(p2k[pt], st);
        if (r != TA_OK) return r;
      }
      if (nchunks) {
        k_select<0><<<(unsigned)nchunks, SEL_THREADS, 0, st>>>(sp);
        k_select<1><<<(unsigned)nchunks, SEL_THREADS, 0, st>>>(sp);
        k_select<2><<<(unsigned)nchunks, SEL_THREADS, 0, st>>>(sp);
        k_labels<<<(unsigned)nchunks, SEL_THREADS, 0, st>>>(sp);
      }
      if (exch && hist_bytes) TA_CU(cudaMemsetAsync(xh, 0, hist_bytes, st));
      if (nx) k_hist<0><<<xsel_chunks, SEL_THREADS, 0, st>>>(xsp);
      break;
    case TA_PHASE_SEL1:
    case TA_PHASE_SEL2:
      if (nx) {
        if (phase == TA_PHASE_SEL1) k_pick<0><<<nx, SEL_THREADS, 0, st>>>(xp);
        else k_pick<1><<<nx, SEL_THREADS, 0, st>>>(xp);
      }
      if (exch && hist_bytes) TA_CU(cudaMemsetAsync(xh, 0, hist_bytes, st));
      if (nx) {
        if (phase == TA_PHASE_SEL1) k_hist<1><<<xsel_chunks, SEL_THREADS, 0, st>>>(xsp);
        else k_hist<2><<<xsel_chunks, SEL_THREADS, 0, st>>>(xsp);
      }
      break;
    case TA_PHASE_LABELS: {
      if (nx) {
        k_pick<2><<<nx, SEL_THREADS, 0, st>>>(xp);
        k_labels<<<xsel_chunks, SEL_THREADS, 0, st>>>(xsp);
      }
      ta_status r = launch_ef(efk, st);  // every label is final here
      if (r != TA_OK) return r;
      break;
    }
    default:
      return fail(TA_ERR_INVALID, "unknown phase " + std::to_string(phase));
  }
  TA_CU(cudaGetLastError());
  return TA_OK;
}

// phase < 0: the whole step (no spanning tensors allowed); phase 0..4: one
// phase of a sharded step (TA_PHASE_*), exch the caller's exchange buffer.
ta_status run_step(const ta_tensor* ts, int nT, const ta_group* groups, uint64_t seed,
                   uint8_t* ws, size_t ws_bytes, cudaStream_t st, void* const* ev = nullptr,
                   int phase = -1, uint8_t* exch = nullptr, size_t chunk_bytes = 0,
                   size_t hist_bytes = 0, int mode = 0, const ta_dynamic* dyn = nullptr) {
  // mode 0: upload the descriptor table and run; 1: upload only (prepare);
  // 2: run on a prepared table with device-advanced step values (no copies)
  auto mark = [&](int i) -> cudaError_t {
    if (ev && ev[i]) return cudaEventRecord((cudaEvent_t)ev[i], st);
    return cudaSuccess;
  };
  std::vector<int64_t> bp = cs_bpads(ts, nT);
  Layout L = layout_for(nT, bp);
  if (ws_bytes < L.total)
    return fail(TA_ERR_WORKSPACE, "workspace too small: need " + std::to_string(L.total) +
                                      " bytes, got " + std::to_string(ws_bytes));
  bool any_span = false;
  for (int i = 0; i < nT; ++i) {
    if (!is_spanning(ts[i])) continue;
    any_span = true;
    const int64_t gb = ts[i].global_blocks ? ts[i].global_blocks : cdiv(ts[i].numel, BS);
    if (phase < 0)
      return fail(TA_ERR_INVALID, "TA_M_SPANNING tensors need the phased step (ta_step_phase)");
    if (ts[i].exch_chunk_off < 0 || ts[i].exch_hist_off < 0 ||
        (size_t)(ts[i].exch_chunk_off + xchunk_elems(gb)) * sizeof(double) > chunk_bytes ||
        (size_t)(ts[i].exch_hist_off + kXHistElems) * sizeof(uint32_t) > hist_bytes)
      return fail(TA_ERR_WORKSPACE, "tensor " + std::to_string(i) +
                                        ": exchange slot outside the exchange regions");
  }
  if (any_span && (!exch || chunk_bytes % 16))
    return fail(TA_ERR_INVALID, "exchange buffer missing or chunk region not 16-byte sized");
  std::vector<uint8_t> host(L.lists + L.list_stride * kMaxLists, 0);
  DevTensor* H = reinterpret_cast<DevTensor*>(host.data() + L.table);
  std::vector<int32_t> cs_list;
  int ci = 0;
  for (int i = 0; i < nT; ++i) {
    if (ts[i].numel == 0) {
      memset(&H[i], 0, sizeof(DevTensor));
      continue;
    }
    H[i] = make_dev(ts[i], groups[ts[i].group], seed);
    if (is_costate(ts[i])) {
      const CsSlot& s = L.cs[ci++];
      H[i].part = reinterpret_cast<float*>(ws + s.part);
      H[i].ratios = reinterpret_cast<float*>(ws + s.ratios);
      H[i].hist = reinterpret_cast<uint32_t*>(ws + s.hist);
      H[i].sel = reinterpret_cast<uint32_t*>(ws + s.sel);
      H[i].alpha_new = reinterpret_cast<float*>(ws + s.alpha);
      H[i].chunk = reinterpret_cast<double*>(ws + s.chunk);
      if (s.efd) H[i].efd = reinterpret_cast<float*>(ws + s.efd);
      cs_list.push_back(i);
      if (is_spanning(ts[i])) {
        H[i].xchunk = reinterpret_cast<double*>(exch) + ts[i].exch_chunk_off;
        H[i].xhist = reinterpret_cast<uint32_t*>(exch + chunk_bytes) + ts[i].exch_hist_off;
      }
    }
  }
  // launch lists: pass 1 by (mk, vk, pt, uni), pass 2 by pt, select chunks
  std::vector<std::pair<P1Key, LaunchList>> p1;
  auto p1_list = [&](P1Key k) -> LaunchList& {
    for (auto& e : p1)
      if (e.first.mk == k.mk && e.first.vk == k.vk && e.first.pt == k.pt &&
          e.first.uni == k.uni && e.first.table == k.table)
        return e.second;
    p1.push_back({k, LaunchList()});
    p1.back().second.beg.push_back(0);
    return p1.back().second;
  };
  LaunchList p2[2];
  p2[0].beg.push_back(0);
  p2[1].beg.push_back(0);
  LaunchList sel, alist, xsel, xalist, xlist, efl;  // x*: spanning tensors
  efl.beg.push_back(0);
  sel.beg.push_back(0);
  alist.beg.push_back(0);
  xsel.beg.push_back(0);
  xalist.beg.push_back(0);
  xlist.beg.push_back(0);
  for (int i = 0; i < nT; ++i) {
    if (ts[i].numel == 0) continue;
    const DevTensor& D = H[i];
    const int pt = ts[i].dtype == TA_BF16 ? 1 : 0;
    const bool oneq = vk_of(ts[i]) == VK_ONEQ;
    P1Key k{mk_of(ts[i]), vk_of(ts[i]), pt, (D.flags & DF_UNI) && oneq, oneq && D.nbits <= 6};
    LaunchList& l = p1_list(k);
    const int64_t tiles = cdiv(D.nblk, TB);
    l.idx.push_back(i);
    l.beg.push_back(l.beg.back() + tiles);
    if (is_costate(ts[i])) {
      p2[pt].idx.push_back(i);
      p2[pt].beg.push_back(p2[pt].beg.back() + tiles);
      LaunchList& sl = is_spanning(ts[i]) ? xsel : sel;
      LaunchList& al = is_spanning(ts[i]) ? xalist : alist;
      sl.idx.push_back(i);
      sl.beg.push_back(sl.beg.back() + D.sel_chunks);
      al.idx.push_back(i);
      al.beg.push_back(al.beg.back() + D.alpha_chunks);
      if (is_spanning(ts[i])) {
        xlist.idx.push_back(i);
        xlist.beg.push_back(xlist.beg.back() + 1);
      }
      if (D.flags & DF_EF) {
        efl.idx.push_back(i);
        efl.beg.push_back(efl.beg.back() + cdiv(D.n, TE));
      }
    }
  }
  // serialise the lists into the host image of the workspace
  int slot = 0;
  auto put = [&](const LaunchList& l, const int64_t** dbeg, const int32_t** didx) {
    uint8_t* base = host.data() + L.lists + L.list_stride * slot;
    memcpy(base, l.beg.data(), l.beg.size() * sizeof(int64_t));
    memcpy(base + (size_t)(nT + 1) * sizeof(int64_t), l.idx.data(),
           l.idx.size() * sizeof(int32_t));
    *dbeg = reinterpret_cast<const int64_t*>(ws + L.lists + L.list_stride * slot);
    *didx = reinterpret_cast<const int32_t*>(ws + L.lists + L.list_stride * slot +
                                             (size_t)(nT + 1) * sizeof(int64_t));
    ++slot;
  };
  uint32_t rk0[10], rk1[10];
  for (int r = 0; r < 10; ++r) {  // Philox key schedule (ta_philox4x32_10)
    rk0[r] = (uint32_t)seed + (uint32_t)r * TA_PHILOX_W0;
    rk1[r] = (uint32_t)(seed >> 32) + (uint32_t)r * TA_PHILOX_W1;
  }
  auto set_rk = [&](KParams& kp) {
    memcpy(kp.rk0, rk0, sizeof(rk0));
    memcpy(kp.rk1, rk1, sizeof(rk1));
  };
  std::vector<KParams> p1k(p1.size());
  uint32_t* status = reinterpret_cast<uint32_t*>(ws + L.status);
  uint32_t* skip = mode == 2 ? status + 1 : nullptr;
  const DevTensor* dT = reinterpret_cast<const DevTensor*>(ws + L.table);
  for (size_t i = 0; i < p1.size(); ++i) {
    KParams& kp = p1k[i];
    put(p1[i].second, &kp.lbeg, &kp.lidx);
    kp.T = dT;
    kp.nl = (int32_t)p1[i].second.idx.size();
    kp.total = p1[i].second.beg.back();
    kp.status = status;
    kp.skip = skip;
    set_rk(kp);
  }
  KParams p2k[2];
  for (int pt = 0; pt < 2; ++pt) {
    put(p2[pt], &p2k[pt].lbeg, &p2k[pt].lidx);
    p2k[pt].T = dT;
    p2k[pt].nl = (int32_t)p2[pt].idx.size();
    p2k[pt].total = p2[pt].beg.back();
    p2k[pt].status = status;
    p2k[pt].skip = skip;
    set_rk(p2k[pt]);
  }
  SelParams sp;
  sp.T = dT;
  sp.skip = skip;
  put(sel, &sp.cbeg, &sp.cidx);
  sp.ncs = (int32_t)sel.idx.size();
  const int64_t nchunks = sel.beg.back();
  SelParams ap;
  ap.T = dT;
  ap.skip = skip;
  put(alist, &ap.cbeg, &ap.cidx);
  ap.ncs = (int32_t)alist.idx.size();
  const int64_t achunks = alist.beg.back();
  SelParams xsp, xap, xp;
  xsp.T = xap.T = xp.T = dT;
  xsp.skip = xap.skip = xp.skip = skip;
  put(xsel, &xsp.cbeg, &xsp.cidx);
  xsp.ncs = (int32_t)xsel.idx.size();
  put(xalist, &xap.cbeg, &xap.cidx);
  xap.ncs = (int32_t)xalist.idx.size();
  put(xlist, &xp.cbeg, &xp.cidx);
  xp.ncs = (int32_t)xlist.idx.size();
  const unsigned nx = (unsigned)xlist.idx.size();
  KParams efk;
  put(efl, &efk.lbeg, &efk.lidx);
  efk.T = dT;
  efk.nl = (int32_t)efl.idx.size();
  efk.total = efl.beg.back();
  efk.status = status;
  efk.skip = skip;
  const unsigned xsel_chunks = (unsigned)xsel.beg.back();
  const unsigned xa_chunks = (unsigned)xalist.beg.back();

  // the descriptor table and the list slots in use; phases after the first
  // of a sharded step run on the table that phase uploaded
  if (mode != 2 && phase <= 0)
    TA_CU(cudaMemcpyAsync(ws + L.table, host.data() + L.table,
                          L.lists + L.list_stride * (size_t)slot - L.table,
                          cudaMemcpyHostToDevice, st));
  if (mode == 1) return TA_OK;
  // the select state (alpha's last-CTA counter first of all) starts each step
  // at zero, wherever a new tensor list put it
  if (L.sel_bytes && (phase < 0 || phase == TA_PHASE_PASS1))
    TA_CU(cudaMemsetAsync(ws + L.sel_block, 0, L.sel_bytes, st));
  if (mode == 2) {
    AdvParams a;
    a.T = reinterpret_cast<DevTensor*>(ws + L.table);
    a.n = nT;
    a.steps = dyn->steps_dev;
    a.table = dyn->bias_table_dev;
    a.tsteps = dyn->table_steps;
    a.lr = dyn->lr_dev;
    a.gscale = dyn->grad_scale_dev;
    a.finf = dyn->found_inf_dev;
    a.skip = skip;
    a.status = status;
    k_advance<<<(unsigned)std::max<int64_t>(1, cdiv(nT, 256)), 256, 0, st>>>(a);
    TA_CU(cudaGetLastError());
  }
  if (phase >= 0) return run_phase(phase, p1, p1k, p2k, ap, achunks, sp, nchunks, xap, xa_chunks,
                                   xsp, xsel_chunks, xp, nx, efk, exch, chunk_bytes, hist_bytes,
                                   st);
  TA_CU(mark(0));
  for (size_t i = 0; i < p1.size(); ++i) {
    const P1Key& k = p1[i].first;
    ta_status r = dispatch_p1(k.mk, k.vk, k.pt, k.uni, k.table, p1k[i], st);
    if (r != TA_OK) return r;
  }
  TA_CU(mark(1));
  if (!cs_list.empty()) {
    k_alpha<<<(unsigned)achunks, FIN_THREADS, 0, st>>>(ap);
    TA_CU(cudaGetLastError());
    TA_CU(mark(2));
    if (p2k[0].total) {
      ta_status r = launch_p2<0>(p2k[0], st);
      if (r != TA_OK) return r;
    }
    if (p2k[1].total) {
      ta_status r = launch_p2<1>(p2k[1], st);
      if (r != TA_OK) return r;
    }
    TA_CU(mark(3));
    k_select<0><<<(unsigned)nchunks, SEL_THREADS, 0, st>>>(sp);
    k_select<1><<<(unsigned)nchunks, SEL_THREADS, 0, st>>>(sp);
    k_select<2><<<(unsigned)nchunks, SEL_THREADS, 0, st>>>(sp);
    k_labels<<<(unsigned)nchunks, SEL_THREADS, 0, st>>>(sp);
    TA_CU(cudaGetLastError());
    ta_status r = launch_ef(efk, st);
    if (r != TA_OK) return r;
  } else {
    TA_CU(mark(2));
    TA_CU(mark(3));
  }
  TA_CU(mark(4));
  return TA_OK;
}

}  // namespace

extern "C" {

int ta_abi_version(void) { return TA_ABI_VERSION; }

const char* ta_last_error(void) { return g_err.c_str(); }

int64_t ta_state_padded_blocks(int64_t n, int32_t block_size) {
  if (n <= 0 || block_size <= 0) return 0;
  return cdiv(cdiv(n, block_size), TB) * TB;
}

size_t ta_workspace_size(const ta_tensor* tensors, int32_t n_tensors) {
  if (n_tensors < 0 || (n_tensors > 0 && !tensors)) return 0;
  return layout_for(n_tensors, cs_bpads(tensors, n_tensors)).total;
}

ta_status ta_step(const ta_tensor* tensors, int32_t n_tensors, const ta_group* groups,
                  int32_t n_groups, uint64_t seed, void* workspace_dev, size_t workspace_bytes,
                  void* stream) {
  g_err.clear();
  if (n_tensors < 0 || (n_tensors > 0 && (!tensors || !groups)) || n_groups < 0)
    return fail(TA_ERR_INVALID, "bad tensor / group arrays");
  if (!workspace_dev || !aligned16(workspace_dev))
    return fail(TA_ERR_INVALID, "workspace must be a 16-byte aligned device pointer");
  for (int i = 0; i < n_tensors; ++i) {
    ta_status r = validate(tensors[i], i, n_groups, groups);
    if (r != TA_OK) return r;
  }
  return run_step(tensors, n_tensors, groups, seed, (uint8_t*)workspace_dev, workspace_bytes,
                  (cudaStream_t)stream);
}

ta_status ta_step_profiled(const ta_tensor* tensors, int32_t n_tensors, const ta_group* groups,
                           int32_t n_groups, uint64_t seed, void* workspace_dev,
                           size_t workspace_bytes, void* stream, void* const* phase_events) {
  g_err.clear();
  if (n_tensors < 0 || (n_tensors > 0 && (!tensors || !groups)) || n_groups < 0)
    return fail(TA_ERR_INVALID, "bad tensor / group arrays");
  if (!workspace_dev || !aligned16(workspace_dev))
    return fail(TA_ERR_INVALID, "workspace must be a 16-byte aligned device pointer");
  for (int i = 0; i < n_tensors; ++i) {
    ta_status r = validate(tensors[i], i, n_groups, groups);
    if (r != TA_OK) return r;
  }
  return run_step(tensors, n_tensors, groups, seed, (uint8_t*)workspace_dev, workspace_bytes,
                  (cudaStream_t)stream, phase_events);
}

ta_status ta_exchange_layout(const int64_t* global_blocks, int32_t n, int64_t* chunk_off,
                             int64_t* hist_off, size_t* chunk_bytes, size_t* hist_bytes) {
  g_err.clear();
  if (n < 0 || (n > 0 && (!global_blocks || !chunk_off || !hist_off)) || !chunk_bytes ||
      !hist_bytes)
    return fail(TA_ERR_INVALID, "bad arguments");
  int64_t c = 0, h = 0;
  for (int i = 0; i < n; ++i) {
    if (global_blocks[i] <= 0) return fail(TA_ERR_INVALID, "global_blocks must be > 0");
    chunk_off[i] = c;
    c += xchunk_elems(global_blocks[i]);
    hist_off[i] = h;
    h += kXHistElems;
  }
  *chunk_bytes = al256((size_t)c * sizeof(double));
  *hist_bytes = al256((size_t)h * sizeof(uint32_t));
  return TA_OK;
}

ta_status ta_step_phase(const ta_tensor* tensors, int32_t n_tensors, const ta_group* groups,
                        int32_t n_groups, uint64_t seed, void* workspace_dev,
                        size_t workspace_bytes, void* exchange_dev, size_t chunk_bytes,
                        size_t hist_bytes, int32_t phase, void* stream) {
  g_err.clear();
  if (n_tensors < 0 || (n_tensors > 0 && (!tensors || !groups)) || n_groups < 0)
    return fail(TA_ERR_INVALID, "bad tensor / group arrays");
  if (!workspace_dev || !aligned16(workspace_dev))
    return fail(TA_ERR_INVALID, "workspace must be a 16-byte aligned device pointer");
  if (phase < TA_PHASE_PASS1 || phase > TA_PHASE_LABELS)
    return fail(TA_ERR_INVALID, "phase must be one of TA_PHASE_*");
  if (exchange_dev && !aligned16(exchange_dev))
    return fail(TA_ERR_INVALID, "exchange buffer must be 16-byte aligned");
  for (int i = 0; i < n_tensors; ++i) {
    ta_status r = validate(tensors[i], i, n_groups, groups);
    if (r != TA_OK) return r;
  }
  return run_step(tensors, n_tensors, groups, seed, (uint8_t*)workspace_dev, workspace_bytes,
                  (cudaStream_t)stream, nullptr, phase, (uint8_t*)exchange_dev, chunk_bytes,
                  hist_bytes);
}

ta_status ta_plan_prepare(const ta_tensor* tensors, int32_t n_tensors, const ta_group* groups,
                          int32_t n_groups, uint64_t seed, void* workspace_dev,
                          size_t workspace_bytes, void* stream) {
  g_err.clear();
  if (n_tensors < 0 || (n_tensors > 0 && (!tensors || !groups)) || n_groups < 0)
    return fail(TA_ERR_INVALID, "bad tensor / group arrays");
  if (!workspace_dev || !aligned16(workspace_dev))
    return fail(TA_ERR_INVALID, "workspace must be a 16-byte aligned device pointer");
  for (int i = 0; i < n_tensors; ++i) {
    ta_tensor t = tensors[i];
    if (t.step == 0) t.step = 1;  // the device advances the counts
    ta_status r = validate(t, i, n_groups, groups);
    if (r != TA_OK) return r;
  }
  return run_step(tensors, n_tensors, groups, seed, (uint8_t*)workspace_dev, workspace_bytes,
                  (cudaStream_t)stream, nullptr, -1, nullptr, 0, 0, 1, nullptr);
}

ta_status ta_step_prepared(const ta_tensor* tensors, int32_t n_tensors, const ta_group* groups,
                           int32_t n_groups, uint64_t seed, void* workspace_dev,
                           size_t workspace_bytes, const ta_dynamic* dyn, void* stream) {
  g_err.clear();
  if (n_tensors < 0 || (n_tensors > 0 && (!tensors || !groups)) || n_groups < 0)
    return fail(TA_ERR_INVALID, "bad tensor / group arrays");
  if (!workspace_dev || !aligned16(workspace_dev))
    return fail(TA_ERR_INVALID, "workspace must be a 16-byte aligned device pointer");
  if (!dyn || !dyn->steps_dev || !dyn->bias_table_dev || dyn->table_steps <= 0)
    return fail(TA_ERR_INVALID, "ta_dynamic needs steps_dev and a bias table");
  for (int i = 0; i < n_tensors; ++i) {
    ta_tensor t = tensors[i];
    if (t.step == 0) t.step = 1;
    if (t.flags & TA_M_SPANNING)
      return fail(TA_ERR_UNSUPPORTED, "the prepared step does not take split tensors");
    ta_status r = validate(t, i, n_groups, groups);
    if (r != TA_OK) return r;
  }
  return run_step(tensors, n_tensors, groups, seed, (uint8_t*)workspace_dev, workspace_bytes,
                  (cudaStream_t)stream, nullptr, -1, nullptr, 0, 0, 2, dyn);
}

ta_status ta_read_status(void* workspace_dev, int32_t clear, uint32_t* status_out,
                         void* stream) {
  if (!workspace_dev || !status_out) return fail(TA_ERR_INVALID, "null argument");
  cudaStream_t st = (cudaStream_t)stream;
  uint32_t v = 0;
  TA_CU(cudaMemcpyAsync(&v, workspace_dev, 4, cudaMemcpyDeviceToHost, st));
  if (clear) TA_CU(cudaMemsetAsync(workspace_dev, 0, 4, st));
  TA_CU(cudaStreamSynchronize(st));
  *status_out = v;
  return TA_OK;
}

size_t ta_aux_workspace_size(int64_t n) {
  if (n <= 0) return 0;
  const int64_t bpad = cdiv(cdiv(n, BS), TB) * TB;
  ta_tensor t;
  memset(&t, 0, sizeof(t));
  t.numel = n;
  t.flags = TA_M_COSTATE;
  const size_t step_ws = layout_for(1, {bpad}).total;
  // padded 1Q copies for the single-tensor seams: idx + hdr
  return al256(step_ws) + al256((size_t)bpad * BS) + al256((size_t)bpad * 4);
}

ta_status ta_v_init(int64_t n, int32_t block_size, uint8_t* idx_dev, uint16_t* hdr_dev,
                    void* stream) {
  g_err.clear();
  if (n <= 0 || !idx_dev || !hdr_dev) return fail(TA_ERR_INVALID, "bad arguments");
  if (block_size != BS) return fail(TA_ERR_UNSUPPORTED, "only block_size 128 is built");
  // compress_v_logscale(full(1e-30), stochastic_round=False): min == max
  const float l = ta_logf(1e-30f);
  const uint16_t h = ta_f32_to_f16(l);
  const int64_t nblk = cdiv(n, BS);
  const int grid = (int)std::min<int64_t>(cdiv(nblk * BS, 256), (int64_t)sm_count() * 8);
  k_v_init<<<grid, 256, 0, (cudaStream_t)stream>>>(idx_dev, hdr_dev, nblk, h);
  TA_CU(cudaGetLastError());
  return TA_OK;
}

ta_status ta_v_decode(const uint8_t* idx_dev, const uint16_t* hdr_dev, int64_t n,
                      int32_t block_size, int32_t v_bits, float* v_out_dev, void* stream) {
  g_err.clear();
  if (n <= 0 || !idx_dev || !hdr_dev || !v_out_dev) return fail(TA_ERR_INVALID, "bad arguments");
  if (block_size != BS) return fail(TA_ERR_UNSUPPORTED, "only block_size 128 is built");
  if (v_bits < 1 || v_bits > 8) return fail(TA_ERR_INVALID, "v_bits out of range");
  const int grid = (int)std::min<int64_t>(cdiv(n, 256), (int64_t)sm_count() * 8);
  k_v_decode<<<grid, 256, 0, (cudaStream_t)stream>>>(idx_dev, hdr_dev, n,
                                                      (float)(1 << v_bits), v_out_dev);
  TA_CU(cudaGetLastError());
  return TA_OK;
}

ta_status ta_v_update(const uint8_t* idx_dev, const uint16_t* hdr_dev, const void* grad_dev,
                      int32_t grad_dtype, int64_t n, int32_t block_size, int32_t v_bits,
                      double beta2, const float* uniforms_dev, uint64_t seed,
                      uint32_t tensor_id, uint32_t step, uint8_t* out_idx_dev,
                      uint16_t* out_hdr_dev, float* v_out_dev, void* workspace_dev,
                      size_t workspace_bytes, void* stream) {
  g_err.clear();
  if (n <= 0 || !idx_dev || !hdr_dev || !grad_dev || !out_idx_dev || !out_hdr_dev ||
      !workspace_dev)
    return fail(TA_ERR_INVALID, "bad arguments");
  if (workspace_bytes < ta_aux_workspace_size(n))
    return fail(TA_ERR_WORKSPACE, "workspace too small (ta_aux_workspace_size)");
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t nblk = cdiv(n, BS), bpad = cdiv(nblk, TB) * TB;
  uint8_t* ws = (uint8_t*)workspace_dev;
  const size_t step_ws = al256(layout_for(1, {bpad}).total);
  uint8_t* pidx = ws + step_ws;
  uint16_t* phdr = reinterpret_cast<uint16_t*>(pidx + al256((size_t)bpad * BS));
  TA_CU(cudaMemcpyAsync(pidx, idx_dev, (size_t)nblk * BS, cudaMemcpyDeviceToDevice, st));
  TA_CU(cudaMemcpyAsync(phdr, hdr_dev, (size_t)nblk * 4, cudaMemcpyDeviceToDevice, st));
  ta_tensor t;
  memset(&t, 0, sizeof(t));
  t.grad_dev = grad_dev;
  t.numel = n;
  t.dtype = grad_dtype;
  t.group = 0;
  t.flags = TA_V_ONEQ | TA_NO_PARAM;
  t.tensor_id = tensor_id;
  t.step = step ? step : 1;
  t.v_idx_dev = pidx;
  t.v_hdr_dev = phdr;
  t.sr_uniforms_dev = uniforms_dev;
  t.v_out_dev = v_out_dev;
  ta_group g;
  memset(&g, 0, sizeof(g));
  g.beta2 = beta2;
  g.beta1 = 0.9;
  g.bc1 = g.bc2 = 1.0f;
  g.block_size = block_size;
  g.v_bits = v_bits;
  g.null_pct = 0.1;
  g.amp_pct = 0.9;
  ta_status r = validate(t, 0, 1, &g);
  if (r != TA_OK) return r;
  r = run_step(&t, 1, &g, seed, ws, step_ws, st);
  if (r != TA_OK) return r;
  TA_CU(cudaMemcpyAsync(out_idx_dev, pidx, (size_t)nblk * BS, cudaMemcpyDeviceToDevice, st));
  TA_CU(cudaMemcpyAsync(out_hdr_dev, phdr, (size_t)nblk * 4, cudaMemcpyDeviceToDevice, st));
  return TA_OK;
}

ta_status ta_costate_decode(const uint8_t* labels_dev, const uint8_t* signs_dev,
                            const float* norms_dev, const uint16_t* amp_dev,
                            const float* alpha_dev, const void* grad_dev, int32_t grad_dtype,
                            int64_t n, int32_t block_size, float* m_out_dev, void* stream) {
  g_err.clear();
  if (n <= 0 || !labels_dev || !signs_dev || !norms_dev || !amp_dev || !alpha_dev ||
      !grad_dev || !m_out_dev)
    return fail(TA_ERR_INVALID, "bad arguments");
  if (block_size != BS) return fail(TA_ERR_UNSUPPORTED, "only block_size 128 is built");
  const int grid = (int)std::min<int64_t>(cdiv(n, 256), (int64_t)sm_count() * 8);
  const float sq = (float)std::sqrt((double)block_size);
  if (grad_dtype == TA_BF16)
    k_cs_decode<1><<<grid, 256, 0, (cudaStream_t)stream>>>(
        labels_dev, signs_dev, norms_dev, amp_dev, alpha_dev, grad_dev, n, sq, m_out_dev);
  else
    k_cs_decode<0><<<grid, 256, 0, (cudaStream_t)stream>>>(
        labels_dev, signs_dev, norms_dev, amp_dev, alpha_dev, grad_dev, n, sq, m_out_dev);
  TA_CU(cudaGetLastError());
  return TA_OK;
}

ta_status ta_costate_encode(const float* delta_dev, int64_t n, int32_t block_size,
                            uint8_t* signs_dev, float* norms_dev, uint16_t* amp_dev,
                            void* stream) {
  g_err.clear();
  if (n <= 0 || !delta_dev || !signs_dev || !norms_dev || !amp_dev)
    return fail(TA_ERR_INVALID, "bad arguments");
  if (block_size != BS) return fail(TA_ERR_UNSUPPORTED, "only block_size 128 is built");
  const int64_t nblk = cdiv(n, BS);
  const int64_t warps = cdiv(nblk, 4);
  const int grid = (int)std::min<int64_t>(cdiv(warps * 32, 256), (int64_t)sm_count() * 8);
  k_cs_encode<<<grid, 256, 0, (cudaStream_t)stream>>>(delta_dev, n, nblk,
                                                      (float)std::sqrt((double)block_size),
                                                      signs_dev, norms_dev, amp_dev);
  TA_CU(cudaGetLastError());
  return TA_OK;
}

ta_status ta_thresholds(const float* ratios_dev, int64_t n_blocks, double null_pct,
                        double amp_pct, float* tau_dev, uint8_t* labels_dev,
                        void* workspace_dev, size_t workspace_bytes, void* stream) {
  g_err.clear();
  if (n_blocks <= 0 || !ratios_dev || !tau_dev || !workspace_dev)
    return fail(TA_ERR_INVALID, "bad arguments");
  const int64_t bpad = cdiv(n_blocks, TB) * TB;
  Layout L = layout_for(1, {bpad});
  if (workspace_bytes < L.total) return fail(TA_ERR_WORKSPACE, "workspace too small");
  cudaStream_t st = (cudaStream_t)stream;
  uint8_t* ws = (uint8_t*)workspace_dev;
  std::vector<uint8_t> host(L.lists + L.list_stride, 0);
  DevTensor* H = reinterpret_cast<DevTensor*>(host.data() + L.table);
  memset(H, 0, sizeof(DevTensor));
  H->n = n_blocks * BS;
  H->nblk = n_blocks;
  H->bpad = bpad;
  threshold_ranks(n_blocks, null_pct, amp_pct, &H->k_lo, &H->k_hi);
  H->ratios = const_cast<float*>(ratios_dev);
  H->hist = reinterpret_cast<uint32_t*>(ws + L.cs[0].hist);
  H->sel = reinterpret_cast<uint32_t*>(ws + L.cs[0].sel);
  H->alpha_new = reinterpret_cast<float*>(ws + L.cs[0].alpha);
  H->lab = labels_dev;
  H->sel_chunks = (int32_t)cdiv(n_blocks, SEL_CHUNK);
  int64_t* beg = reinterpret_cast<int64_t*>(host.data() + L.lists);
  beg[0] = 0;
  beg[1] = H->sel_chunks;
  int32_t* idx = reinterpret_cast<int32_t*>(host.data() + L.lists + 2 * sizeof(int64_t));
  idx[0] = 0;
  TA_CU(cudaMemcpyAsync(ws + L.table, host.data() + L.table, host.size() - L.table,
                        cudaMemcpyHostToDevice, st));
  // zero histograms / counters, set the ranks (what k_alpha does in a step)
  TA_CU(cudaMemsetAsync(ws + L.cs[0].hist, 0, (size_t)3 * 2 * HBINS * 4, st));
  uint32_t sel0[16] = {0};
  sel0[SEL_RLO] = (uint32_t)H->k_lo;
  sel0[SEL_RHI] = (uint32_t)H->k_hi;
  TA_CU(cudaMemcpyAsync(ws + L.cs[0].sel, sel0, sizeof(sel0), cudaMemcpyHostToDevice, st));
  SelParams sp;
  sp.T = reinterpret_cast<const DevTensor*>(ws + L.table);
  sp.cbeg = reinterpret_cast<const int64_t*>(ws + L.lists);
  sp.cidx = reinterpret_cast<const int32_t*>(ws + L.lists + 2 * sizeof(int64_t));
  sp.ncs = 1;
  const unsigned nch = (unsigned)H->sel_chunks;
  k_select<0><<<nch, SEL_THREADS, 0, st>>>(sp);
  k_select<1><<<nch, SEL_THREADS, 0, st>>>(sp);
  k_select<2><<<nch, SEL_THREADS, 0, st>>>(sp);
  if (labels_dev) k_labels<<<nch, SEL_THREADS, 0, st>>>(sp);
  TA_CU(cudaGetLastError());
  TA_CU(cudaMemcpyAsync(tau_dev, ws + L.cs[0].alpha + 4, 8, cudaMemcpyDeviceToDevice, st));
  return TA_OK;
}

}  // extern "C"

// ---- ta_v_update_noalloc: ta_v_update's scratch in a static device array --
// One instance per device (module globals are per context). Its device
// address is looked up on every call, with the caller's device current
// (cudaGetSymbolAddress allocates nothing); the first call that sees a new
// address -- the first call on a device, or the first after the module was
// loaded again by a context reset -- zeroes the whole array once.
static __device__ __align__(256) uint8_t g_noalloc_scratch[TA_V_UPDATE_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of the static scratch on the current device (return code
// checked); zeroes the array on `st` when the address is new.
ta_status noalloc_scratch(cudaStream_t st, void** out) {
  int dev = -1;
  TA_CU(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return fail(TA_ERR_UNSUPPORTED, "device ordinal " + std::to_string(dev) +
                                        " above the static scratch table");
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || !p)
    return fail(TA_ERR_CUDA, std::string("cudaGetSymbolAddress(static scratch): ") +
                                 cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] != p) {
    TA_CU(cudaMemsetAsync(p, 0, TA_V_UPDATE_NOALLOC_SCRATCH_BYTES, st));
    g_noalloc_ptr[dev] = p;
  }
  *out = p;
  return TA_OK;
}
// 1 when the hardware pair rounding of (x, -x) differs from the portable one.
__device__ __forceinline__ unsigned long long bf16_mismatch(float x) {
  const uint32_t sw = (uint32_t)ta_f32_to_bf16(x) | ((uint32_t)ta_f32_to_bf16(-x) << 16);
  return bf16x2_rn(x, -x) != sw;
}
__global__ void __launch_bounds__(256) k_selftest_fast_math(unsigned long long* out) {
  unsigned long long me = 0, nm = 0, nr = 0, ers = 0, erc = 0, nb = 0;
  const uint64_t lo = 0x00800000u, hi = 0x7f800000u;  // the normal binary32 numbers
  for (uint64_t u = lo + blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; u < hi;
       u += (uint64_t)gridDim.x * blockDim.x) {
    const float x = __uint_as_float((uint32_t)u);
    const float le = ta_logf_core(x, 0);
    if (u + 1 < hi && ta_logf_core(__uint_as_float((uint32_t)u + 1u), 0) < le) ++nm;
    if (le >= -69.3f) {
      const float la = __fmul_rn(lg2_approx(x), LN2_F);
      const unsigned long long d =
          (unsigned long long)__double_as_longlong(fabs((double)la - (double)le));
      me = d > me ? d : me;
    }
    if (u < 0x7e800000u) {  // 1/x normal
      const float y0 = rcp_approx(x);
      const float y = __fmaf_rn(__fmaf_rn(-x, y0, 1.0f), y0, y0);
      if (__float_as_uint(y) != __float_as_uint(__frcp_rn(x))) ++nr;
      const double rc = fabs((double)y0 * (double)x - 1.0);  // relative error of the estimate
      const unsigned long long rcb = (unsigned long long)__double_as_longlong(rc);
      erc = rcb > erc ? rcb : erc;
    }
    nb += bf16_mismatch(x);
    const double rs = fabs((double)rsqrt_approx(x) * sqrt((double)x) - 1.0);
    const unsigned long long rsb = (unsigned long long)__double_as_longlong(rs);
    ers = rsb > ers ? rsb : ers;
  }
  // the rest of the non-NaN patterns for the bf16 rounding: zeros,
  // subnormals and infinity
  for (uint32_t u = blockIdx.x * blockDim.x + threadIdx.x; u <= lo;
       u += gridDim.x * blockDim.x)
    nb += bf16_mismatch(__uint_as_float(u < lo ? u : hi));
  atomicMax(&out[0], me);
  atomicAdd(&out[1], nm);
  atomicAdd(&out[2], nr);
  atomicMax(&out[3], ers);
  atomicMax(&out[4], erc);
  atomicAdd(&out[5], nb);
}

}  // namespace

extern "C" {

ta_status ta_selftest_fast_math(uint64_t* out_dev, void* stream) {
  g_err.clear();
  if (!out_dev) return fail(TA_ERR_INVALID, "null argument");
  k_selftest_fast_math<<<sm_count() * 8, 256, 0, (cudaStream_t)stream>>>(
      reinterpret_cast<unsigned long long*>(out_dev));
  TA_CU(cudaGetLastError());
  return TA_OK;
}

ta_status ta_selftest_wait_timeout(uint64_t limit_ns, uint32_t* status_dev,
                                   uint64_t* out_dev, void* stream) {
  g_err.clear();
  if (!status_dev || !out_dev) return fail(TA_ERR_INVALID, "null argument");
  if (limit_ns == 0 || limit_ns > WAIT_LIMIT_NS)
    return fail(TA_ERR_INVALID, "limit_ns must be in (0, 2e9]");
  k_selftest_wait<<<1, NTHR, 0, (cudaStream_t)stream>>>(
      limit_ns, status_dev, reinterpret_cast<unsigned long long*>(out_dev));
  TA_CU(cudaGetLastError());
  return TA_OK;
}

ta_status ta_v_update_noalloc(const uint8_t* idx_dev, const uint16_t* hdr_dev,
                              const void* grad_dev, int32_t grad_dtype, int64_t n,
                              int32_t block_size, int32_t v_bits, double beta2,
                              const float* uniforms_dev, uint64_t seed, uint32_t tensor_id,
                              uint32_t step, uint8_t* out_idx_dev, uint16_t* out_hdr_dev,
                              float* v_out_dev, void* stream) {
  g_err.clear();
  if (n > TA_V_UPDATE_NOALLOC_MAX_N)
    return fail(TA_ERR_UNSUPPORTED,
                "n = " + std::to_string(n) + " exceeds the static scratch limit of " +
                    std::to_string(TA_V_UPDATE_NOALLOC_MAX_N) +
                    " elements (TA_V_UPDATE_NOALLOC_MAX_N); use ta_v_update with a workspace");
  if (n > 0 && ta_aux_workspace_size(n) > TA_V_UPDATE_NOALLOC_SCRATCH_BYTES)
    return fail(TA_ERR_UNSUPPORTED, "n = " + std::to_string(n) +
                                        " needs more scratch than the static array holds");
  void* scratch = nullptr;
  if (n > 0) {
    const ta_status r = noalloc_scratch((cudaStream_t)stream, &scratch);
    if (r != TA_OK) return r;
    // the status word (first 4 bytes) reports this call only
    TA_CU(cudaMemsetAsync(scratch, 0, 4, (cudaStream_t)stream));
  }
  return ta_v_update(idx_dev, hdr_dev, grad_dev, grad_dtype, n, block_size, v_bits, beta2,
                     uniforms_dev, seed, tensor_id, step, out_idx_dev, out_hdr_dev, v_out_dev,
                     scratch, TA_V_UPDATE_NOALLOC_SCRATCH_BYTES, stream);
}

ta_status ta_v_update_noalloc_status(int32_t clear, uint32_t* status_out, void* stream) {
  g_err.clear();
  if (!status_out) return fail(TA_ERR_INVALID, "null status_out");
  void* scratch = nullptr;
  const ta_status r = noalloc_scratch((cudaStream_t)stream, &scratch);
  if (r != TA_OK) return r;
  return ta_read_status(scratch, clear, status_out, stream);
}

}  // extern "C"
