// Host-side planning / launching of the tcgen05 flash-attention kernel (attention.cu).
#pragma once

#include <cstring>
#include <cuda_fp16.h>

#include "common.h"

namespace dlm {

// Strided view of a [B, H, S, 64] tensor: element (b, h, s, d) is at ptr + b*sb + h*sh + s*ss + d.
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
};

struct AttnOp {
  CUtensorMap tmQ, tmK, tmV;
  AttnParams p;
  int grid = 0;
};

int attn_plan(AttnOp* op, int B, int H, int Sq, int Sk, int Dh, float scale, const AttnTensor& q,
              const AttnTensor& k, const AttnTensor& v, const AttnTensor& o);
int attn_launch(const AttnOp& op, cudaStream_t s);
int attn_prepare_kernels();

}  // namespace dlm
