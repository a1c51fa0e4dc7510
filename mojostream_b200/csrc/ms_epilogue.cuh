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
// normalisation already applied).  Rows written earlier in the same launch
// (the persistent decode kernel) are read through L2 (ld.global.cg): the L1
// of another SM may still hold an older copy of the line.
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
        const size_t off = kv_row_offset(p.kv.block_table, p.kv.bt_stride, p.kv.page, p.kv.cap,
                                         p.kv.circular, p.seq[m], p.pos[m], p.kv.kv_dim);
        float* pool = td.dst == 1 ? p.kv.k : p.kv.v;
        kv_put(pool, p.kv.bf16, off + td.col_lo + g, a);
        kv_put(pool, p.kv.bf16, off + td.col_hi + g, b);
      }
      break;
    }
    default:
      break;
  }
}

// Inputs of epilogue_row that do not depend on the projection's sums, loaded
// before the main loop so their global-memory latency overlaps it:
//   kEpiResid : the residual values of columns c, c + 8 (a, b)
//   kEpiQKV   : the tile descriptor, the destination (Q row, or K / V pool
//               and row offset) and cos / sin of the RoPE angle (a, b)
struct EpiPrefetch {
  float a, b;
  float* dst;
  size_t off;
  QkvTile td;
};

__device__ __forceinline__ void epilogue_prefetch(const GemvParams& p, int tile, int g, int m,
                                                  EpiPrefetch& e) {
  e.a = e.b = 0.f;
  e.dst = nullptr;
  if (p.epi == kEpiResid) {
    const float* r = p.resid + (size_t)m * p.ldr + tile * kTileN + g;
    e.a = __ldcg(r);
    e.b = __ldcg(r + 8);
  } else if (p.epi == kEpiQKV) {
    e.td = p.tiles[tile];
    const int pos = p.pos[m];
    if (e.td.rope_i0 >= 0) {
      const float th = (float)pos * p.inv_freq[e.td.rope_i0 + g];
      e.a = cosf(th);
      e.b = sinf(th);
    }
    if (e.td.dst == 0) {
      e.dst = p.q_out;
      e.off = (size_t)m * p.ldq;
    } else {
      e.off = kv_row_offset(p.kv.block_table, p.kv.bt_stride, p.kv.page, p.kv.cap, p.kv.circular,
                            p.seq[m], pos, p.kv.kv_dim);
      e.dst = e.td.dst == 1 ? p.kv.k : p.kv.v;
    }
  }
}

// epilogue_row with the inputs of epilogue_prefetch (same arithmetic).
__device__ __forceinline__ void epilogue_row_pre(const GemvParams& p, int tile, int g, int m,
                                                 float v0, float v1, float inv_res,
                                                 const EpiPrefetch& e, float& sq_out) {
  switch (p.epi) {
    case kEpiResid: {
      const int c = tile * kTileN + g;
      const float a = (e.a * p.resid_ple) * inv_res + p.scale * v0;
      const float b = (e.b * p.resid_ple) * inv_res + p.scale * v1;
      float* o = p.out + (size_t)m * p.ldo + c;
      o[0] = a;
      o[8] = b;
      sq_out = a * a + b * b;
      break;
    }
    case kEpiQKV: {
      const float s = e.td.dst == 0 ? p.sq : (e.td.dst == 1 ? p.sk : p.sv);
      float a = s * v0, b = s * v1;
      if (e.td.rope_i0 >= 0) {
        const float ra = a * e.a - b * e.b;
        const float rb = a * e.b + b * e.a;
        a = ra;
        b = rb;
      }
      const int bf = e.td.dst != 0 && p.kv.bf16;
      kv_put(e.dst, bf, e.off + e.td.col_lo + g, a);
      kv_put(e.dst, bf, e.off + e.td.col_hi + g, b);
      break;
    }
    default:
      epilogue_row(p, tile, g, m, v0, v1, inv_res, sq_out);
      break;
  }
}

}  // namespace ms
