// Kernel 2: per-row merge, exact scoring and the draw (one CTA per row).
//
// Merges the candidate sets of a row's streaming units with the row's penalised ids
// (scored here in IEEE double exactly as src/runtime/sampling.ts:26-30 does), orders
// them by (logit/T desc, id asc) exactly as the reference's stable sort
// (src/runtime/sampling.ts:33-35), normalises with the full-vocabulary sum
// (src/runtime/sampling.ts:36-42: the streamed part comes from kernel 1's per-unit
// (max, sum) partials) and runs top-k, min-p, typical-p, top-p and the seeded draw
// (src/runtime/sampling.ts:44-64).  Temperature 0 is the argmax of the penalised logits
// with the lowest id on ties (src/runtime/sampling.ts:31,92-96 and
// src/webgpu/decode-greedy.ts:181-184).
#include "gs_device.cuh"
#include "gs_block.cuh"
#include "gs_filter.cuh"
#include "gs_internal.cuh"
#include "../../include/gsampler.h"

namespace gs {

struct FinShared {
  unsigned flags;
  int n_allowed;
  int n_c;
  int n_ent;
  float raw_m;
  double raw_s;
  double uniform;
  int s_int[4];
  double red_d[32];
  int red_i[32];
  float red_f[32];
  unsigned hist[256];
  int sel_digit;
  int sel_above;
  int sel_binc;
  int fill_base;
  int n_sort;
  unsigned long long min_pack;
  int rec_nc;
  float tok_raw;
};

__device__ __forceinline__ bool mask_allows(const uint32_t* mrow, uint32_t id) {
  return (__ldg(mrow + (id >> 5)) >> (id & 31)) & 1u;
}

// Entries (twice: all scored entries, then those that can reach the top k), the filter
// work arrays (work_cap each) and the history / pack scratch.
size_t finalize_smem_bytes(int hist_cap, int ent_cap, int pack_cap, int work_cap) {
  const size_t r1 = std::max<size_t>(static_cast<size_t>(hist_cap) * 4, static_cast<size_t>(pack_cap) * 8);
  const size_t work = (static_cast<size_t>(work_cap) * (4 + 8 + 8 + 8 + 4 + 4 + 1) + 15) & ~static_cast<size_t>(15);
  return 2 * static_cast<size_t>(ent_cap) * sizeof(Ent) + work + ((r1 + 15) & ~static_cast<size_t>(15)) + 64;
}

template <int DT>
__global__ void __launch_bounds__(kFinalizeMaxThreads) finalize_kernel(const __grid_constant__ FinalizeArgs A) {
  extern __shared__ __align__(16) unsigned char dsm[];
  __shared__ FinShared F;
  const int row = blockIdx.x, tid = threadIdx.x, bs = blockDim.x;
  const RowPlan* pp = A.plans ? A.plans + row : &A.plan0;
  const int mode = pp->mode;
  if (mode == kModeLarge) return;
  const bool greedy = mode == kModeGreedy;
  const double T = pp->temperature;
  const int S = A.splits;

  // ---- shared memory carve-up ----
  unsigned char* p = dsm;
  Ent* ent_all = reinterpret_cast<Ent*>(p);  // every scored entry (normaliser)
  p += static_cast<size_t>(A.ent_cap) * sizeof(Ent);
  Ent* ent = reinterpret_cast<Ent*>(p);      // those that can reach the top k, sorted
  p += static_cast<size_t>(A.ent_cap) * sizeof(Ent);
  const int wc = A.work_cap;
  FilterWork w;
  w.cp = reinterpret_cast<double*>(p);
  p += wc * 8;
  w.cum = reinterpret_cast<double*>(p);
  p += wc * 8;
  w.skey = reinterpret_cast<unsigned long long*>(p);
  p += wc * 8;
  w.cid = reinterpret_cast<uint32_t*>(p);
  p += wc * 4;
  w.sval = reinterpret_cast<uint32_t*>(p);
  p += wc * 4;
  w.pos = reinterpret_cast<int*>(p);
  p += wc * 4;
  w.flg = p;
  p += wc;
  p = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(p) + 15) & ~static_cast<uintptr_t>(15));
  unsigned char* r1 = p;
  w.red_d = F.red_d;
  w.red_i = F.red_i;
  w.s_int = F.s_int;
  w.s_flags = &F.flags;

  const int32_t state = A.mask_state ? A.mask_state[row] : -1;
  const bool has_mask = A.mask_table != nullptr && state >= 0 && state < A.mask_states;
  const uint32_t* mrow = has_mask ? A.mask_table + static_cast<int64_t>(state) * A.mask_words : nullptr;
  const unsigned char* rowbase =
      A.logits ? static_cast<const unsigned char*>(A.logits) + static_cast<int64_t>(row) * A.row_stride * (DT == GS_DTYPE_F32 ? 4 : 2)
               : nullptr;
  // Sources of the row's units: the streaming pass's statistics and packs, or (merge of
  // a vocabulary-sharded row) the gathered shard records, one per shard.
  const bool part_mode = A.shard_mode == 1, merge_mode = A.shard_mode == 2;
  auto rec_of = [&](int u) -> const unsigned char* {
    return A.records + (static_cast<int64_t>(u) * gridDim.x + row) * A.rec_bytes;
  };
  auto unit_stat = [&](int u) -> const UnitStat& {
    return merge_mode ? *reinterpret_cast<const UnitStat*>(rec_of(u)) : A.stats[static_cast<int64_t>(row) * S + u];
  };
  auto unit_pack = [&](int u, int j) -> unsigned long long {
    return merge_mode ? reinterpret_cast<const unsigned long long*>(rec_of(u) + sizeof(UnitStat))[j]
                      : A.cands[(static_cast<int64_t>(row) * S + u) * A.kcap + j];
  };
  unsigned char* my_rec = part_mode ? A.records + static_cast<int64_t>(row) * A.rec_bytes : nullptr;

  // ---- 0. unit partials (the units spread over the threads: rows can have many) ----
  {
    unsigned fl = 0;
    int na = 0, nc = 0;
    float rm = -INFINITY, um = -INFINITY;
    for (int u = tid; u < S; u += bs) {
      const UnitStat& st = unit_stat(u);
      fl |= st.flags;
      na += st.n_allowed;
      nc += st.n_cand;
      rm = fmaxf(rm, st.raw_m);
      um = fmaxf(um, st.m);
    }
    if (tid == 0) F.flags = 0;
    __syncthreads();
    if (fl) atomicOr(&F.flags, fl);
    na = block_sum_i(na, F.red_i);
    nc = block_sum_i(nc, F.red_i);
    rm = block_max_f(rm, F.red_f);
    double rs = 0.0;
    if (A.want_raw) {
      for (int u = tid; u < S; u += bs) {
        const UnitStat& st = unit_stat(u);
        if (st.raw_m > -INFINITY) rs = __dadd_rn(rs, __dmul_rn(st.raw_s, exp(static_cast<double>(st.raw_m) - static_cast<double>(rm))));
      }
      rs = block_sum_d(rs, F.red_d);
    }
    if (part_mode) {
      // the shard's combined (max, sum): the merge combines shards the same way
      const float m = block_max_f(um, F.red_f);
      double sm = 0.0;
      for (int u = tid; u < S; u += bs) {
        const UnitStat& st = unit_stat(u);
        if (st.m > -INFINITY)
          sm = __dadd_rn(sm, __dmul_rn(st.s, exp2(__dmul_rn(static_cast<double>(st.m) - static_cast<double>(m), pp->a2))));
      }
      sm = block_sum_d(sm, F.red_d);
      if (tid == 0) {
        UnitStat* h = reinterpret_cast<UnitStat*>(my_rec);
        h->m = m;
        h->s = m > -INFINITY ? sm : 0.0;
        h->raw_m = rm;
        h->raw_s = rs;
        h->n_allowed = na;
      }
    }
    if (tid == 0) {
      fl = F.flags;
      if (has_mask && na == 0 && !part_mode) fl |= GS_FLAG_ERR_DEADEND;
      if (greedy) fl |= GS_FLAG_GREEDY;
      F.flags = fl;
      F.n_allowed = na;
      F.n_c = nc;
      F.n_ent = 0;
      F.n_sort = 0;
      F.min_pack = ~0ull;
      F.rec_nc = 0;
      F.raw_m = rm;
      F.raw_s = rs;
    }
    __syncthreads();
  }

  // ---- 1. penalty history: distinct ids with counts, scored exactly ----
  if (merge_mode && !(F.flags & GS_FLAG_ERRORS)) {
    // the shards scored their own penalised ids; slot (shard, j) keeps a fixed position
    const int hc = A.rec_hcap;
    for (int i = tid; i < S * hc; i += bs) {
      const int u = i / hc, j = i - u * hc;
      const unsigned char* r = rec_of(u) + sizeof(UnitStat) + 8ll * A.rec_kcap;
      const uint32_t id = reinterpret_cast<const uint32_t*>(r + 8ll * hc)[j];
      ent_all[i] = id == 0xffffffffu ? Ent{-INFINITY, 0xffffffffu, 0xffffffffu}
                                     : Ent{reinterpret_cast<const double*>(r)[j], id, 1u};
    }
    if (tid == 0) F.n_ent = S * hc;
    __syncthreads();
  } else if (!(F.flags & GS_FLAG_ERRORS)) {
    int64_t hl = A.history_len ? A.history_len[row] : 0;
    if (hl > A.history_stride) hl = A.history_stride;
    if (hl < 0) hl = 0;
    if (hl > 0) {
      uint32_t* hs = reinterpret_cast<uint32_t*>(r1);
      // with counts: 64-bit words id << 32 | occurrences, sorted the same way
      unsigned long long* hw = reinterpret_cast<unsigned long long*>(r1);
      const int32_t* hcn = A.history_count ? A.history_count + static_cast<int64_t>(row) * A.history_stride : nullptr;
      const int h2 = pow2_ceil(static_cast<int>(hl));
      const int32_t* h = A.history + static_cast<int64_t>(row) * A.history_stride;
      if (hcn) {
        for (int i = tid; i < h2; i += bs)
          hw[i] = i < hl ? (static_cast<unsigned long long>(static_cast<uint32_t>(h[i])) << 32) |
                               static_cast<uint32_t>(max(hcn[i], 1))
                         : ~0ull;
        __syncthreads();
        bitonic_sort_u64(hw, h2);
      } else {
        for (int i = tid; i < h2; i += bs) hs[i] = i < hl ? static_cast<uint32_t>(h[i]) : 0xffffffffu;
        __syncthreads();
        bitonic_sort_u32(hs, h2);
      }
      auto id_at = [&](int i) -> uint32_t { return hcn ? static_cast<uint32_t>(hw[i] >> 32) : hs[i]; };
      const double rp = pp->repetition_penalty, pres = pp->presence_penalty, freq = pp->frequency_penalty;
      // entry i belongs to sorted history position i (a fixed slot, so the normaliser's
      // summation order does not depend on thread timing); unused slots have kind ~0
      for (int i = tid; i < hl; i += bs) {
        const uint32_t v = id_at(i);  // global id (negative ids are >= 2^31 here)
        const int64_t lv = static_cast<int64_t>(v) - A.vocab_offset;  // local to this call's logits
        Ent e{-INFINITY, 0xffffffffu, 0xffffffffu};
        float x = 0.0f;
        const bool first = lv >= 0 && lv < A.vocab && !(i > 0 && id_at(i - 1) == v);
        if (first && !(has_mask && !mask_allows(mrow, static_cast<uint32_t>(lv)))) {  // masked: -inf either way
          double cnt = 0.0;
          for (int j = i; j < hl && id_at(j) == v; ++j) cnt += hcn ? static_cast<double>(hw[j] & 0xffffffffu) : 1.0;
          x = load_logit(rowbase, DT, lv);
          if (A.softcap != 0.0f) x = softcap(x, A.softcap, A.inv_softcap);
          if (!(x < INFINITY)) atomicOr(&F.flags, GS_FLAG_ERR_NONFINITE);  // NaN or +inf
          const double xp = penalise(static_cast<double>(x), cnt, rp, pres, freq);
          e = Ent{greedy ? xp : __ddiv_rn(xp, T), v, 1u};
        }
        ent_all[i] = e;
        if (part_mode) {
          unsigned char* r = my_rec + sizeof(UnitStat) + 8ll * A.rec_kcap;
          reinterpret_cast<double*>(r)[i] = e.key;
          reinterpret_cast<uint32_t*>(r + 8ll * A.rec_hcap)[i] = e.id;
          reinterpret_cast<float*>(r + 12ll * A.rec_hcap)[i] = x;
        }
      }
      if (tid == 0) F.n_ent = static_cast<int>(hl);
    }
    if (part_mode) {
      unsigned char* r = my_rec + sizeof(UnitStat) + 8ll * A.rec_kcap;
      for (int i = static_cast<int>(hl) + tid; i < A.rec_hcap; i += bs) reinterpret_cast<uint32_t*>(r + 8ll * A.rec_hcap)[i] = 0xffffffffu;
    }
    __syncthreads();
  }

  // ---- 2. streamed candidates of the units (top k over all units) ----
  const int k = greedy ? 1 : pp->k_eff;
  if (!(F.flags & GS_FLAG_ERRORS)) {
    const int nc = F.n_c;
    unsigned long long my_min = ~0ull;  // smallest unit pack this thread adds
    auto add_pack = [&](unsigned long long v) {
      if (part_mode) {  // the shard's top k go to its record
        reinterpret_cast<unsigned long long*>(my_rec + sizeof(UnitStat))[atomicAdd(&F.rec_nc, 1)] = v;
        return;
      }
      const float x = pack_value(v);
      const uint32_t id = pack_id(v);
      const int slot = atomicAdd(&F.n_ent, 1);
      ent_all[slot] = Ent{greedy ? static_cast<double>(x) : __ddiv_rn(static_cast<double>(x), T), id, 0u};
      my_min = v < my_min ? v : my_min;
    };
    if (nc > k) {
      unsigned long long* buf = reinterpret_cast<unsigned long long*>(r1);
      const int np = S * A.kcap;
      for (int i = tid; i < np; i += bs) {
        const int u = i / A.kcap, j = i - u * A.kcap;
        buf[i] = j < unit_stat(u).n_cand ? unit_pack(u, j) : 0ull;
      }
      __syncthreads();
      unsigned long long prefix, mask;
      select_threshold(buf, np, k, F.hist, &F.sel_digit, &F.sel_above, &F.sel_binc, prefix, mask);
      for (int i = tid; i < np; i += bs) {
        const unsigned long long v = buf[i];
        if (v != 0ull && (v & mask) >= prefix) add_pack(v);
      }
    } else {
      for (int i = tid; i < S * A.kcap; i += bs) {
        const int u = i / A.kcap, j = i - u * A.kcap;
        if (j < unit_stat(u).n_cand) add_pack(unit_pack(u, j));
      }
    }
    if (my_min != ~0ull) atomicMin(&F.min_pack, my_min);
    __syncthreads();
  }
  if (part_mode) {  // the record is complete: the rest runs in gs_shard_merge
    if (tid == 0) {
      UnitStat* h = reinterpret_cast<UnitStat*>(my_rec);
      h->n_cand = F.rec_nc;
      h->flags = F.flags;
      h->pad = A.want_raw ? 1 : 0;  // bit 0: raw sums recorded
    }
    return;
  }

  // ---- 3. exact order of the entries that can reach the top k ----
  // With k streamed candidates kept, an entry below the k-th of them has at least k
  // entries before it; only the others are sorted (all still count in the normaliser).
  const int n_all = F.n_ent;
  if (!(F.flags & GS_FLAG_ERRORS)) {
    double thr = -INFINITY;
    if (F.n_c >= k && F.min_pack != ~0ull) {
      const double x = static_cast<double>(pack_value(F.min_pack));
      thr = greedy ? x : __ddiv_rn(x, T);
    }
    for (int i = tid; i < n_all; i += bs) {
      const Ent e = ent_all[i];
      if (e.kind != 0xffffffffu && e.key >= thr) ent[atomicAdd(&F.n_sort, 1)] = e;
    }
    __syncthreads();
    const int ns = F.n_sort;
    const int n2 = pow2_ceil(ns > 0 ? ns : 1);
    for (int i = ns + tid; i < n2; i += bs) ent[i] = Ent{-INFINITY, 0xffffffffu, 0xffffffffu};
    __syncthreads();
    bitonic_sort_ent(ent, n2);
  }

  uint32_t tok = 0xffffffffu;
  int n_final = 0;
  if (!(F.flags & GS_FLAG_ERRORS)) {
    const int n_ent = F.n_sort;
    if (greedy) {
      // argmax over the whole vocabulary: all -inf -> id 0 (sampling.ts:92-96)
      if (n_ent == 0 || ent[0].key == -INFINITY) {
        tok = 0;
      } else {
        tok = ent[0].id;
      }
      if (tid == 0) {
        w.cid[0] = tok;
        w.cp[0] = 1.0;
      }
      n_final = 1;
    } else {
      const int K = pp->top_k;
      int nC = n_ent < K ? n_ent : K;
      // Fewer allowed ids than topK: the remaining slots are -inf ids (masked ones and
      // -inf logits) in ascending id order, exactly as the stable sort leaves them.
      if (has_mask && n_ent < K && F.n_allowed < A.vocab) {
        // masked ids in ascending order, up to K of them
        int* mids = w.pos;
        const int nwords = static_cast<int>((A.vocab + 31) >> 5);
        if (tid == 0) F.fill_base = 0;
        __syncthreads();
        for (int w0 = 0; w0 < nwords && F.fill_base < K; w0 += bs) {
          const int wi = w0 + tid;
          uint32_t zero = 0;
          if (wi < nwords) {
            zero = ~__ldg(mrow + wi);
            if (wi == nwords - 1 && (A.vocab & 31)) zero &= (1u << (A.vocab & 31)) - 1u;
          }
          const int c = __popc(zero);
          // exclusive scan of c over the block
          int incl = c;
          for (int o = 1; o < 32; o <<= 1) {
            const int u = __shfl_up_sync(kFullMask, incl, o);
            if ((tid & 31) >= o) incl += u;
          }
          if ((tid & 31) == 31) F.red_i[tid >> 5] = incl;
          __syncthreads();
          int base = F.fill_base;
          for (int ww = 0; ww < (tid >> 5); ++ww) base += F.red_i[ww];
          base += incl - c;
          for (uint32_t z = zero; z; z &= z - 1) {
            if (base < K) mids[base] = wi * 32 + __ffs(z) - 1;
            ++base;
          }
          __syncthreads();
          if (tid == bs - 1) F.fill_base = base;
          __syncthreads();
        }
        const int n_masked = F.fill_base < K ? F.fill_base : K;
        // merge the -inf tail of ent with the masked ids by id
        if (tid == 0) {
          int j0 = 0;
          while (j0 < n_ent && ent[j0].key > -INFINITY) ++j0;
          int a = j0, b = 0, o = j0;
          // ent[j0, n_ent) are -inf entries sorted by id; merge into w.cum..w.skey
          // (2·work_cap·8 bytes = work_cap entries, unused at this point)
          Ent* tail = reinterpret_cast<Ent*>(w.cum);
          int t = 0;
          while (o < K && (a < n_ent || b < n_masked)) {
            if (b >= n_masked || (a < n_ent && ent[a].id < static_cast<uint32_t>(mids[b]))) {
              tail[t++] = ent[a++];
            } else {
              tail[t++] = Ent{-INFINITY, static_cast<uint32_t>(mids[b++]), 2u};
            }
            ++o;
          }
          for (int i = 0; i < t; ++i) ent[j0 + i] = tail[i];
          F.s_int[0] = j0 + t;
        }
        __syncthreads();
        nC = F.s_int[0];
      }
      const double M = ent[0].key;
      if (M == -INFINITY) {
        if (tid == 0) F.flags |= GS_FLAG_ERR_NONFINITE;  // every logit -inf: outside the domain
      } else {
        // full-vocabulary normaliser: streamed units + every penalised id
        double part = 0.0;
        for (int u = tid; u < S; u += bs) {
          const UnitStat& st = unit_stat(u);
          if (st.m > -INFINITY)
            part = __dadd_rn(part, __dmul_rn(st.s, exp(__dsub_rn(__ddiv_rn(static_cast<double>(st.m), T), M))));
        }
        for (int i = tid; i < n_all; i += bs)
          if (ent_all[i].kind == 1u) part = __dadd_rn(part, exp(__dsub_rn(ent_all[i].key, M)));
        const double total = block_sum_d(part, F.red_d);
        for (int i = tid; i < nC; i += bs) {
          w.cid[i] = ent[i].id;
          w.cp[i] = __ddiv_rn(exp(__dsub_rn(ent[i].key, M)), total);
        }
        if (tid == 0) {
          double r;
          if (A.uniforms) {
            r = A.uniforms[row];
          } else {
            double st = A.rng_state[row];
            r = seeded_next(&st);
            A.rng_state[row] = st;
          }
          F.uniform = r;
        }
        __syncthreads();
        tok = filter_and_draw(w, nC, pp->min_p, pp->typical_p, pp->top_p, F.uniform, &n_final);
      }
    }
  }
  __syncthreads();

  // ---- outputs ----
  const unsigned fl = F.flags;
  const bool err = (fl & GS_FLAG_ERRORS) != 0;
  if (merge_mode && A.logprob && !err) {
    // the drawn id's soft-capped logit, from the shard that holds it
    if (tid == 0) F.tok_raw = __int_as_float(0x7fffffff);
    __syncthreads();
    const int per = A.rec_kcap + A.rec_hcap;
    for (int i = tid; i < S * per; i += bs) {
      const int u = i / per, j = i - u * per;
      if (j < A.rec_kcap) {
        if (j < unit_stat(u).n_cand && pack_id(unit_pack(u, j)) == tok) F.tok_raw = pack_value(unit_pack(u, j));
      } else {
        const unsigned char* r = rec_of(u) + sizeof(UnitStat) + 8ll * A.rec_kcap;
        const int jj = j - A.rec_kcap;
        if (reinterpret_cast<const uint32_t*>(r + 8ll * A.rec_hcap)[jj] == tok)
          F.tok_raw = reinterpret_cast<const float*>(r + 12ll * A.rec_hcap)[jj];
      }
    }
    __syncthreads();
  }
  if (tid == 0) {
    A.ids[row] = err ? -1 : static_cast<int32_t>(tok);
    if (A.flags) A.flags[row] = fl;
    if (A.cand_count) A.cand_count[row] = err ? 0 : n_final;
    if (A.logprob) {
      double lp = NAN;
      if (!err) {
        float x;
        if (merge_mode) {
          // NaN when the drawn id is a masked filler (no shard holds its logit) or a shard
          // recorded no raw sums
          x = F.tok_raw;
          for (int u = 0; u < S; ++u)
            if (!(unit_stat(u).pad & 1)) x = __int_as_float(0x7fffffff);
        } else {
          x = load_logit(rowbase, DT, tok);
          if (A.softcap != 0.0f) x = softcap(x, A.softcap, A.inv_softcap);
        }
        lp = __dsub_rn(__dsub_rn(static_cast<double>(x), static_cast<double>(F.raw_m)), log(F.raw_s));
      }
      A.logprob[row] = lp;
    }
  }
  if (A.cand_ids) {
    // final candidates in draw order; unused slots are -1 / 0 so outputs are fully defined
    const int nw = err ? 0 : (n_final < A.cand_cap ? n_final : A.cand_cap);
    for (int i = tid; i < A.cand_cap; i += bs) {
      A.cand_ids[static_cast<int64_t>(row) * A.cand_cap + i] = i < nw ? static_cast<int32_t>(w.cid[i]) : -1;
      if (A.cand_probs) A.cand_probs[static_cast<int64_t>(row) * A.cand_cap + i] = i < nw ? w.cp[i] : 0.0;
    }
  }
}

cudaError_t launch_finalize(const FinalizeArgs& a, int dtype, int rows, size_t smem, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  // Fewer rows than two per SM: more threads per row shorten each row's chain.  Measured
  // at C3's settings (one B200, merge time): 64 rows 39.2 us with 1024 threads, 35.3 with
  // 512; 128 rows 41.1 / 38.3; 256 rows 44.8 with 256 threads, 39.1 with 512, 74.8 with
  // 1024 (one CTA per SM).  A handful of rows keep 1024.
  const int threads = rows < 32 ? kFinalizeMaxThreads : (rows < 2 * sm_count() ? 512 : kFinalizeThreads);
  if (dtype == GS_DTYPE_F32) {
    const cudaError_t e = cudaFuncSetAttribute(finalize_kernel<GS_DTYPE_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    finalize_kernel<GS_DTYPE_F32><<<rows, threads, smem, st>>>(a);
  } else {
    const cudaError_t e = cudaFuncSetAttribute(finalize_kernel<GS_DTYPE_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    finalize_kernel<GS_DTYPE_BF16><<<rows, threads, smem, st>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace gs
