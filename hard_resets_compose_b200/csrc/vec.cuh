// NPL consecutive neurons per lane: one float (NPL = 1) or one float4 (NPL = 4,
// 16-byte aligned) per load and store.
#pragma once

namespace lifb {

template <int NPL>
struct Vec {
    float v[NPL];
};

template <int NPL>
__device__ __forceinline__ Vec<NPL> ld_vec(const float *p)
{
    Vec<NPL> r;
    if constexpr (NPL == 4) {
        float4 t = *reinterpret_cast<const float4 *>(p);
        r.v[0] = t.x; r.v[1] = t.y; r.v[2] = t.z; r.v[3] = t.w;
    } else {
        r.v[0] = *p;
    }
    return r;
}

template <int NPL>
__device__ __forceinline__ void st_vec(float *p, const Vec<NPL> &a)
{
    if constexpr (NPL == 4) {
        *reinterpret_cast<float4 *>(p) = make_float4(a.v[0], a.v[1], a.v[2], a.v[3]);
    } else {
        *p = a.v[0];
    }
}

}  // namespace lifb
