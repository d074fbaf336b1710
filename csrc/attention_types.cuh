// Parameters shared by the paged cascade attention kernels (attention.cu:
// mma.sync decode and prefill; attention_tc.cu: tcgen05 prefill).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"

namespace braid {

struct AttnParams {
  const __nv_bfloat16* q;  // [T, Hq, D] unrotated
  const __nv_bfloat16* kv; // layer pool [P, 2, Hkv, PS, D]
  __nv_bfloat16* out;      // [T, Hq*D]
  const int* qo_indptr;
  const int* positions;
  const int* seg_indptr;
  const int* seg_page_indptr;
  const int* seg_offset;
  const int* seg_len;
  const int* seg_pos0;
  const int* seg_delta;
  const int* page_ids;
  const float* cos;
  const float* sin;
  float scale_log2;
  int use_rope;
  int rope_len;
  int Hq, Hkv, G, PS;
  int num_pages;    // pages of the KV pool (checked build)
  int num_splits;
  float* part_o;    // [T, Hq, splits, D]
  float* part_lse;  // [T, Hq, splits]
  int* counters;    // [T * Hkv] split arrival counters, kept at zero between launches
  unsigned long long* trace;  // optional per-CTA phase timestamps (profiling)
  unsigned long long* tc_trace;  // tcgen05 prefill: 128 timestamps per CTA (profiling)
  unsigned long long* span;   // optional launch span (profiling)
  PrefetchArgs pf;            // decode: the next GEMM's weight to pull into L2 (tensor map tmP)
  int pf_early;
  int cta_rows;               // tcgen05 prefill: query rows per CTA (256 = two Q tiles, or 128)
  int use_tc;                 // prefill launch: the tcgen05 kernel (attention_tc.cu), else mma.sync               // decode: issue that prefetch with the first K/V tiles (else after the last)
  int kv_evict_first;         // decode: read K/V with the evict-first L2 policy
  // Shared-prefix decode (segments common to a group of sequences are read
  // once for all of them): partials live at split index split_base + split
  // of split_stride slots per (token, head).  The shared pass (prefill kernel,
  // partial_only) fills slots [0, split_base of the decode pass); the decode
  // pass merges its own splits with those slots for the group's sequences.
  int split_stride;           // partial slots per (token, head); 0: num_splits
  int split_base;             // first slot of this launch's splits
  int partial_only;           // prefill kernel: publish partials, do not merge
  const int* seq_nsh;         // decode: 1 for sequences of the shared-prefix group (nullptr: none)
};

constexpr float LOG2E = 1.4426950408889634f;
constexpr int KT = 64;  // keys per tile

}  // namespace braid
