// Host-side planning / launching of the tcgen05 flash-attention kernel (attention.cu).
#pragma once

#include <cstring>
#include <cuda_fp16.h>

#include "common.h"

namespace dlm {

// Strided view of a [B, H, S, Dh] tensor: element (b, h, s, d) is at ptr + b*sb + h*sh + s*ss + d.
struct AttnTensor {
  const __half* ptr = nullptr;
  long long sb = 0, sh = 0, ss = 0;
};

struct AttnParams {
  int B, H, Sq, Sk;
  float scale_log2;  // softmax scale * log2(e)
  __half* out;
  long long o_sb, o_sh, o_ss;
  int* status;
  // stream-K (sk_ctas > 0, grid == sk_ctas): the groups' KV tile-steps are split evenly over the
  // CTAs; every segment of a group cut between CTAs leaves its normalised O rows (fp16) and
  // (row max, row sum) in slot 2 * cta + (cta holds the group's first tiles ? 1 : 0), and the CTA
  // that finishes the group last (arrival counter part_cnt[group], zero between launches) merges
  // the slots in CTA order.
  int sk_ctas;
  __half* part_o;   // [2 * sk_ctas][256][64]
  float2* part_ml;  // [2 * sk_ctas][256]
  int* part_cnt;    // [groups]
};

struct AttnOp {
  CUtensorMap tmQ, tmK, tmV;
  AttnParams p;
  int grid = 0;
};

// Workspace for stream-K (optional, ws == nullptr keeps one CTA per 256-query block): at least
// attn_workspace_bytes(B, H, Sq) bytes, 256-byte aligned, its first attn_counter_bytes(B, H, Sq)
// bytes zero before the first launch (every launch leaves them zero).  Launches sharing a
// workspace must not overlap on the GPU.
int attn_plan(AttnOp* op, int B, int H, int Sq, int Sk, int Dh, float scale, const AttnTensor& q,
              const AttnTensor& k, const AttnTensor& v, const AttnTensor& o, void* ws = nullptr,
              size_t ws_bytes = 0);
size_t attn_workspace_bytes(int B, int H, int Sq);
size_t attn_counter_bytes(int B, int H, int Sq);
int attn_launch(const AttnOp& op, cudaStream_t s);
int attn_prepare_kernels();

// Wide heads (attention_wide.cu): head_dim a multiple of 64 in [128, 512], one CTA per (batch,
// head, 128-query tile, output slice of dv = Dh or Dh / 2 columns).
struct AttnWideParams {
  int B, H, Sq, Sk, Dh;
  int dv, nsplit;      // output columns per CTA, Dh / dv
  float scale_log2;    // softmax scale * log2(e)
  __half* out;
  long long o_sb, o_sh, o_ss;
  int* status;
};

struct AttnWideOp {
  CUtensorMap tmQ, tmK, tmV;
  AttnWideParams p;
  int grid = 0;
};

int attn_wide_plan(AttnWideOp* op, int B, int H, int Sq, int Sk, int Dh, float scale,
                   const AttnTensor& q, const AttnTensor& k, const AttnTensor& v,
                   const AttnTensor& o);
int attn_wide_launch(const AttnWideOp& op, cudaStream_t s);

}  // namespace dlm
