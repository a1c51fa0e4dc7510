// ms_epilogue.cuh -- the fused epilogues of the Q4 projection kernels.
//
// Reference steps folded into the projection that produces their input
// (src/main.mojo:538-613, src/inference/gemma4_e4b.mojo:459-540):
//   kEpiStore / kEpiAccum : C (+)= s * acc            (matmul_q4_bpack_raw)
//   kEpiResid  : x_out = ple * x * inv_rms(x) + s * acc, i.e. the residual add
//                onto the normalised input (main.mojo:599-600, 612-613), plus
//                the per-tile sums of squares the next RMSNorm needs
//   kEpiSwiGLU : h = up * g * sigmoid(g)  (kernels.mojo:519-532)
//   kEpiQKV    : RoPE on Q / K pairs (kernels.mojo:553-595), then Q to its
//                buffer and K / V into the paged cache (main.mojo:584-592)
#pragma once

#include "ms_common.cuh"
#include "ms_kernels.h"

namespace ms {

// v0 / v1: the finished sums of tile rows g and g + 8 for row m (any input
// normalisation already applied).  Residual rows are read through L2
// (ld.global.cg), never through the non-coherent L1 / texture path.
__device__ __forceinline__ void epilogue_row(const GemvParams& p, int tile, int g, int m,
                                             float v0, float v1, float inv_res,
                                             float& sq_out) {
  switch (p.epi) {
    case kEpiStore:
    case kEpiAccum: {
      float* o = p.out + (size_t)m * p.ldo + tile * kTileN + g;
      float a = p.scale * v0, b = p.scale * v1;
      if (p.epi == kEpiAccum) {
        a = __ldcg(o) + a;
        b = __ldcg(o + 8) + b;
      }
      o[0] = a;
      o[8] = b;
      break;
    }
    case kEpiResid: {
      const int c = tile * kTileN + g;
      const float* r = p.resid + (size_t)m * p.ldr + c;
      const float a = (__ldcg(r) * p.resid_ple) * inv_res + p.scale * v0;
      const float b = (__ldcg(r + 8) * p.resid_ple) * inv_res + p.scale * v1;
      float* o = p.out + (size_t)m * p.ldo + c;
      o[0] = a;
      o[8] = b;
      sq_out = a * a + b * b;
      break;
    }
    case kEpiSwiGLU: {
      const float gt = p.scale * v0, up = p.scale2 * v1;
      const float sig = 1.0f / (1.0f + expf(-gt));
      const float h = up * gt * sig;
      p.out[(size_t)m * p.ldo + tile * 8 + g] = h;
      break;
    }
    case kEpiQKV: {
      const QkvTile td = p.tiles[tile];
      const float s = td.dst == 0 ? p.sq : (td.dst == 1 ? p.sk : p.sv);
      float a = s * v0, b = s * v1;
      if (td.rope_i0 >= 0) {
        const float th = (float)p.pos[m] * p.inv_freq[td.rope_i0 + g];
        const float cs = cosf(th), sn = sinf(th);
        const float ra = a * cs - b * sn;
        const float rb = a * sn + b * cs;
        a = ra;
        b = rb;
      }
      if (td.dst == 0) {
        float* o = p.q_out + (size_t)m * p.ldq;
        o[td.col_lo + g] = a;
        o[td.col_hi + g] = b;
      } else {
        size_t off;
        int bf;
        float* pool = kv_dst(p.kv, td.dst, m, p.seq[m], p.pos[m], off, bf);
        kv_put(pool, bf, off + td.col_lo + g, a);
        kv_put(pool, bf, off + td.col_hi + g, b);
      }
      break;
    }
    default:
      break;
  }
}


}  // namespace ms
