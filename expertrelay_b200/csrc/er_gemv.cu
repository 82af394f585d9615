// er_gemv.cu -- K3a: grouped weight-streaming GEMV for decode-sized groups.
//
// Reference: runtime/qwen_moe.py:345-348 (per expert
// down(silu(gate(x)) * up(x)) through int8_linear / int4_linear) and
// :353-357 (the shared expert), with int8_linear.py:57-66 (fused decode
// kernel: y[i, r] = s_r * sum_j x[i, j] q[r, j]) and int4_linear.py:40-59
// (fused int4: per-group partial sums times the group scale).
//
// Work item = a block of weight rows of one group (all of its tokens). Each
// warp owns kGemvRowsPerWarp weight rows for the whole K range; lanes split K
// in 16-value chunks read with 16-byte (int8) or 8-byte (int4) streaming
// loads, so each weight byte is read from HBM exactly once. The group's
// activations are staged in shared memory as fp32, kGemvMaxTok tokens at a
// time. mode 0 (gate/up): a warp's rows are 4 gate rows and the same 4 up
// rows and the epilogue writes act = silu(g * s_g) * (u * s_u). mode 1 (down):
// 8 rows of the down matrix, y = acc * s_d * routing weight (or * sigmoid gate
// for the shared expert).
#include "er_internal.cuh"

namespace er {

constexpr int kGemvSlab = 1024;  // K values staged per pass

template <int FMT, int MODE, typename XT>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_grouped_kernel(GroupArgs a, int sched,
                                                                       const XT* __restrict__ x,
                                                                       float* act_r,
                                                                       float* act_s,
                                                                       float* __restrict__ out_r,
                                                                       float* __restrict__ out_s) {
  constexpr int R = kGemvRowsPerWarp;
  constexpr int MT = kGemvMaxTok;
  constexpr bool kInt8 = (FMT == ER_FMT_INT8);
  __shared__ __align__(16) float xs[MT * kGemvSlab];
  chain_wait();
  const Plan* P = a.plan;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = P->item_start[sched][P->num_active];
  for (int item = blockIdx.x; item < total; item += gridDim.x) {
    int local = 0;
    const int g = find_item(P, sched, item, &local);
    if (g < 0) break;
    const GroupView v = group_view(a, g);
    // the shared expert is always an int8 record; routed groups use FMT
    if (v.fmt != FMT) continue;
    const RecordGeom geo{v.fmt, a.H, v.inter, a.group};
    const int K = MODE == 0 ? a.H : v.inter;
    const int units = MODE == 0 ? v.inter : a.H;
    const size_t row_bytes = kInt8 ? (size_t)K : (size_t)K / 2;
    const int ngroups = kInt8 ? 1 : K / a.group;

    // this warp's rows: mode 0 -> columns c0..c0+R/2-1 of gate (r < R/2) and of up;
    // mode 1 -> rows c0..c0+R-1 of down
    const int c0 = MODE == 0 ? local * kGemvUnitsGU + warp * (R / 2) : local * kGemvUnitsDN + warp * R;
    const size_t woff0 = geo.weight_offset(MODE == 0 ? 0 : 2), woff1 = geo.weight_offset(1);
    const size_t soff0 = geo.scale_offset(MODE == 0 ? 0 : 2), soff1 = geo.scale_offset(1);
    const size_t zoff0 = geo.zero_offset(MODE == 0 ? 0 : 2), zoff1 = geo.zero_offset(1);
    auto row_of = [&](int r) { return c0 + (MODE == 0 ? (r % (R / 2)) : r); };
    auto upper = [&](int r) { return MODE == 0 && r >= R / 2; };
    bool valid[R];
#pragma unroll
    for (int r = 0; r < R; ++r) valid[r] = row_of(r) < units;
    for (int t0 = 0; t0 < v.rows; t0 += MT) {
      const int mt = min(MT, v.rows - t0);
      float acc[R][MT];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < MT; ++t) acc[r][t] = 0.f;

      for (int k0 = 0; k0 < K; k0 += kGemvSlab) {
        const int sl = min(kGemvSlab, K - k0);
        __syncthreads();
        for (int i = threadIdx.x * 4; i < mt * sl; i += blockDim.x * 4) {
          const int t = i / sl, kk = i - t * sl;
          float4 val;
          if (MODE == 0) {
            const int tok = v.shared ? t0 + t : a.perm_token[v.row0 + t0 + t];
            val = load4(x + (size_t)tok * a.H + k0 + kk);
          } else {
            const float* src = v.shared ? act_s + (size_t)(t0 + t) * v.inter
                                        : act_r + (size_t)(v.row0 + t0 + t) * a.I;
            val = *reinterpret_cast<const float4*>(src + k0 + kk);
          }
          *reinterpret_cast<float4*>(xs + t * kGemvSlab + kk) = val;
        }
        __syncthreads();
        for (int kk = lane * 16; kk < sl; kk += 512) {
          uint32_t wv[R][4];
          float sc[R], zr[R];
#pragma unroll
          for (int r = 0; r < R; ++r) {
            if (kInt8) {
              const uint8_t* wp = v.rec + (upper(r) ? woff1 : woff0) + (size_t)row_of(r) * row_bytes;
              uint4 q = valid[r] ? ld_stream_u4(wp + k0 + kk) : make_uint4(0, 0, 0, 0);
              wv[r][0] = q.x;
              wv[r][1] = q.y;
              wv[r][2] = q.z;
              wv[r][3] = q.w;
            } else {
              const uint8_t* wp = v.rec + (upper(r) ? woff1 : woff0) + (size_t)row_of(r) * row_bytes;
              uint2 q = valid[r] ? ld_stream_u2(wp + (k0 + kk) / 2) : make_uint2(0, 0);
              wv[r][0] = q.x;
              wv[r][1] = q.y;
              const size_t gidx = (size_t)row_of(r) * ngroups + (k0 + kk) / a.group;
              const uint16_t* sp = reinterpret_cast<const uint16_t*>(v.rec + (upper(r) ? soff1 : soff0));
              sc[r] = valid[r] ? half_bits_to_f32(sp[gidx]) : 0.f;
              zr[r] = (FMT == ER_FMT_INT4_ZP && valid[r]) ? (float)(v.rec + (upper(r) ? zoff1 : zoff0))[gidx] : 8.f;
            }
          }
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            if (t < mt) {
              float xv[16];
              const float4* xp = reinterpret_cast<const float4*>(xs + t * kGemvSlab + kk);
#pragma unroll
              for (int q4 = 0; q4 < 4; ++q4) {
                const float4 f = xp[q4];
                xv[4 * q4] = f.x;
                xv[4 * q4 + 1] = f.y;
                xv[4 * q4 + 2] = f.z;
                xv[4 * q4 + 3] = f.w;
              }
              if (kInt8) {
#pragma unroll
                for (int r = 0; r < R; ++r) {
                  float s = acc[r][t];
#pragma unroll
                  for (int wi = 0; wi < 4; ++wi) {
                    float f[4];
                    i8x4_to_f32(wv[r][wi], f);
#pragma unroll
                    for (int j = 0; j < 4; ++j) s = fmaf(f[j], xv[4 * wi + j], s);
                  }
                  acc[r][t] = s;
                }
              } else {
                float xsum = 0.f;
#pragma unroll
                for (int j = 0; j < 16; ++j) xsum += xv[j];
#pragma unroll
                for (int r = 0; r < R; ++r) {
                  float d = 0.f;
#pragma unroll
                  for (int wi = 0; wi < 2; ++wi) {
                    float f[8];
                    u4x8_to_f32(wv[r][wi], f);
#pragma unroll
                    for (int j = 0; j < 8; ++j) d = fmaf(f[j], xv[8 * wi + j], d);
                  }
                  acc[r][t] = fmaf(sc[r], fmaf(-zr[r], xsum, d), acc[r][t]);
                }
              }
            }
          }
        }
      }

      // reduce over lanes; lane (r * MT + t) % 32 writes entry (r, t)
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < MT; ++t)
          if (t < mt) acc[r][t] = warp_sum(acc[r][t]);

      if (MODE == 0) {
#pragma unroll
        for (int c = 0; c < R / 2; ++c) {
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            if (t < mt && valid[c] && lane == ((c * MT + t) & 31)) {
              const int col = c0 + c;
              float gs, us;
              if (kInt8 || v.shared) {
                gs = reinterpret_cast<const float*>(v.rec + soff0)[col];
                us = reinterpret_cast<const float*>(v.rec + soff1)[col];
              } else {
                gs = us = 1.f;  // int4 scales were applied per group
              }
              const float gval = acc[c][t] * gs;
              const float uval = acc[c + R / 2][t] * us;
              float* dst = v.shared ? act_s + (size_t)(t0 + t) * v.inter
                                    : act_r + (size_t)(v.row0 + t0 + t) * a.I;
              dst[col] = silu_f(gval) * uval;
            }
          }
        }
      } else {
#pragma unroll
        for (int r = 0; r < R; ++r) {
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            if (t < mt && valid[r] && lane == ((r * MT + t) & 31)) {
              const int row = c0 + r;
              const float s = (kInt8 || v.shared) ? reinterpret_cast<const float*>(v.rec + soff0)[row] : 1.f;
              const float yv = acc[r][t] * s;
              if (v.shared)
                out_s[(size_t)(t0 + t) * a.H + row] = yv * a.gate_sig[t0 + t];
              else
                out_r[(size_t)(v.row0 + t0 + t) * a.H + row] = yv * a.perm_w[v.row0 + t0 + t];
            }
          }
        }
      }
    }
  }
}

template <int MODE, typename XT>
static int launch_fmt(const GroupArgs& a, int sched, const XT* x, float* act_r, float* act_s,
                      float* out_r, float* out_s, int grid, cudaStream_t st) {
  // the shared expert (int8) is processed by the int8 instance; routed groups by
  // the instance of their format (each instance skips groups of another format)
  if (int rc = launch_chained(gemv_grouped_kernel<ER_FMT_INT8, MODE, XT>, dim3(grid), dim3(kGemvWarps * 32), 0, st,
                              "gemv_grouped_kernel<int8>", a, sched, x, act_r, act_s, out_r, out_s))
    return rc;
  if (a.fmt == ER_FMT_INT4)
    return launch_chained(gemv_grouped_kernel<ER_FMT_INT4, MODE, XT>, dim3(grid), dim3(kGemvWarps * 32), 0, st,
                          "gemv_grouped_kernel<int4>", a, sched, x, act_r, act_s, out_r, out_s);
  if (a.fmt == ER_FMT_INT4_ZP)
    return launch_chained(gemv_grouped_kernel<ER_FMT_INT4_ZP, MODE, XT>, dim3(grid), dim3(kGemvWarps * 32), 0, st,
                          "gemv_grouped_kernel<int4zp>", a, sched, x, act_r, act_s, out_r, out_s);
  return ER_OK;
}

int launch_gemv_grouped(const GroupArgs& a, int sched, int mode, const void* x, int x_dtype, float* act_r,
                        float* act_s, float* out_r, float* out_s, long long items_bound, cudaStream_t st) {
  if (items_bound <= 0) return ER_OK;
  const int grid = (int)(items_bound < 65535 ? items_bound : 65535);
  if (mode == 0) {
    if (x_dtype == ER_DTYPE_BF16)
      return launch_fmt<0, __nv_bfloat16>(a, sched, (const __nv_bfloat16*)x, act_r, act_s, out_r, out_s, grid, st);
    return launch_fmt<0, float>(a, sched, (const float*)x, act_r, act_s, out_r, out_s, grid, st);
  }
  return launch_fmt<1, float>(a, sched, nullptr, act_r, act_s, out_r, out_s, grid, st);
}

}  // namespace er
