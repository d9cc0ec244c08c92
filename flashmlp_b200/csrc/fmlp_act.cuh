// Activation functions and their derivatives, fused into the kernels' epilogues.
// Mirrors the reference's device functions (flashmlp.py:27-46, inline sigmoid :145) and
// the rounding points of its kernels: H = act(Z) is rounded to the input dtype, and the
// silu / sigmoid derivatives are formed from that rounded H (flashmlp.py:227-235).
#pragma once
#include "fmlp_ptx.cuh"

namespace fmlp {

// h = act(z) in fp32 (unrounded).
template <typename T, int ACT>
__device__ __forceinline__ float act_fwd(float z) {
  if constexpr (ACT == kLeakyRelu) {
    return fmaxf(z, 0.01f * z);  // == where(z >= 0, z, 0.01 z) for slope < 1
  } else if constexpr (ACT == kSilu) {
    // z * sigma(z) = z * (0.5 tanh(z/2) + 0.5) = u tanh(u) + u with u = z/2: one multiply,
    // one MUFU op and one FMA (the activation warps are issue-bound next to the SFU)
    const float u = 0.5f * z;
    return fmaf(u, tanh_approx(u), u);
  } else if constexpr (ACT == kSigmoid) {
    return sigmoid_fast(z);
  } else {
    return z;
  }
}

// What the derivative needs from the forward activation of one element.
template <typename T, int ACT>
struct ActState {
  float s;   // sigmoid(z) (silu)
  float hr;  // h rounded to the input dtype (silu, sigmoid)
  bool pos;  // z >= 0 (leaky_relu)
};

// h = act(z), unrounded; records the state act_grad needs.
template <typename T, int ACT>
__device__ __forceinline__ float act_forward(float z, ActState<T, ACT>& st) {
  if constexpr (ACT == kLeakyRelu) {
    st.pos = z >= 0.f;
    return fmaxf(z, 0.01f * z);
  } else if constexpr (ACT == kSilu) {
    st.s = sigmoid_fast(z);
    const float h = z * st.s;
    st.hr = Pack<T>::round(h);
    return h;
  } else if constexpr (ACT == kSigmoid) {
    const float h = sigmoid_fast(z);
    st.hr = Pack<T>::round(h);
    return h;
  } else {
    return z;
  }
}

// dz = dh * act'(z), formed from the rounded h where the reference does so.
template <typename T, int ACT>
__device__ __forceinline__ float act_grad(float dh, const ActState<T, ACT>& st) {
  if constexpr (ACT == kLeakyRelu) {
    return dh * (st.pos ? 1.0f : 0.01f);  // flashmlp.py:33-34, :227-228
  } else if constexpr (ACT == kSilu) {
    return dh * (st.s + st.hr * (1.0f - st.s));  // d_silu(z, h), flashmlp.py:43-46
  } else if constexpr (ACT == kSigmoid) {
    // dh * sig * (1 - sig), sig the rounded h; (1 - sig) is formed in the input dtype
    // as in flashmlp.py:232-233.
    return (dh * st.hr) * Pack<T>::round(1.0f - st.hr);
  } else {
    return dh;
  }
}

// Activates a pair: returns H rounded and packed (z0 in the low half) and records the
// derivative state; the rounded H is read back from the packed word with integer ops.
template <typename T, int ACT>
__device__ __forceinline__ uint32_t act_pair(float z0, float z1, ActState<T, ACT>& s0, ActState<T, ACT>& s1) {
  // the scalar operations of sigmoid_fast and act_forward, two elements per instruction
  float h0, h1;
  if constexpr (ACT == kLeakyRelu) {
    s0.pos = z0 >= 0.f;
    s1.pos = z1 >= 0.f;
    const uint64_t m = mul2(f2(0.01f, 0.01f), f2(z0, z1));
    h0 = fmaxf(z0, f2_lo(m));
    h1 = fmaxf(z1, f2_hi(m));
  } else if constexpr (ACT == kSilu) {
    const uint64_t half = f2(0.5f, 0.5f), z = f2(z0, z1);
    const uint64_t u = mul2(half, z);
    const uint64_t sg = fma2(half, f2(tanh_approx(f2_lo(u)), tanh_approx(f2_hi(u))), half);
    const uint64_t h = mul2(z, sg);
    s0.s = f2_lo(sg), s1.s = f2_hi(sg);
    h0 = f2_lo(h), h1 = f2_hi(h);
  } else if constexpr (ACT == kSigmoid) {
    const uint64_t half = f2(0.5f, 0.5f);
    const uint64_t u = mul2(half, f2(z0, z1));
    const uint64_t sg = fma2(half, f2(tanh_approx(f2_lo(u)), tanh_approx(f2_hi(u))), half);
    h0 = f2_lo(sg), h1 = f2_hi(sg);
  } else {
    h0 = z0;
    h1 = z1;
  }
  const uint32_t p = Pack<T>::pack(h0, h1);
  if constexpr (ACT == kSilu || ACT == kSigmoid) {
    s0.hr = Pack<T>::lo(p);
    s1.hr = Pack<T>::hi(p);
  }
  return p;
}

// What the fused dW schedule keeps per element between its two phases: the factor(s) dH
// is multiplied by, formed from the forward state in phase 1, when the activation warps
// would otherwise wait for dH. grad_from_fac(dh, grad_fac(st)) performs exactly the
// operations of act_grad(dh, st) in the same order, so the results are bit-identical.
template <typename T, int ACT>
struct GradFac {
  float f;  // silu: s + h (1 - s); leaky_relu: 1 or 0.01; sigmoid: the rounded h
  float g;  // sigmoid: (1 - h) rounded to the input dtype
};

template <typename T, int ACT>
__device__ __forceinline__ GradFac<T, ACT> grad_fac(const ActState<T, ACT>& st) {
  if constexpr (ACT == kLeakyRelu) {
    return {st.pos ? 1.0f : 0.01f, 0.f};
  } else if constexpr (ACT == kSilu) {
    return {st.s + st.hr * (1.0f - st.s), 0.f};
  } else if constexpr (ACT == kSigmoid) {
    return {st.hr, Pack<T>::round(1.0f - st.hr)};
  } else {
    return {1.0f, 0.f};
  }
}

template <typename T, int ACT>
__device__ __forceinline__ float grad_from_fac(float dh, const GradFac<T, ACT>& a) {
  if constexpr (ACT == kLeakyRelu || ACT == kSilu) {
    return dh * a.f;
  } else if constexpr (ACT == kSigmoid) {
    return (dh * a.f) * a.g;
  } else {
    return dh;
  }
}

// Activates a pair (packed rounded H returned) and records the factors dH is multiplied by.
template <typename T, int ACT>
__device__ __forceinline__ uint32_t act_pair_fac(float z0, float z1, GradFac<T, ACT>& a0, GradFac<T, ACT>& a1) {
  ActState<T, ACT> s0, s1;
  const uint32_t p = act_pair<T, ACT>(z0, z1, s0, s1);
  if constexpr (ACT == kSilu) {  // grad_fac's s + h (1 - s), two elements per instruction
    const uint64_t sg = f2(s0.s, s1.s);
    const uint64_t f = fma2(f2(s0.hr, s1.hr), sub2(f2(1.0f, 1.0f), sg), sg);
    a0.f = f2_lo(f), a1.f = f2_hi(f);
    a0.g = a1.g = 0.f;
  } else {
    a0 = grad_fac<T, ACT>(s0);
    a1 = grad_fac<T, ACT>(s1);
  }
  return p;
}

// dz = dh * act'(z) for a pair from the recorded factors, rounded and packed.
template <typename T, int ACT>
__device__ __forceinline__ uint32_t grad_pair_fac(float dh0, float dh1, const GradFac<T, ACT>& a0,
                                                  const GradFac<T, ACT>& a1) {
  if constexpr (ACT == kLeakyRelu || ACT == kSilu) {  // grad_from_fac, two elements per instruction
    const uint64_t d = mul2(f2(dh0, dh1), f2(a0.f, a1.f));
    return Pack<T>::pack(f2_lo(d), f2_hi(d));
  } else if constexpr (ACT == kSigmoid) {
    const uint64_t d = mul2(mul2(f2(dh0, dh1), f2(a0.f, a1.f)), f2(a0.g, a1.g));
    return Pack<T>::pack(f2_lo(d), f2_hi(d));
  } else {
    return Pack<T>::pack(grad_from_fac<T, ACT>(dh0, a0), grad_from_fac<T, ACT>(dh1, a1));
  }
}

// dz = dh * act'(z) for a pair, rounded and packed.
template <typename T, int ACT>
__device__ __forceinline__ uint32_t grad_pair(float dh0, float dh1, const ActState<T, ACT>& s0,
                                              const ActState<T, ACT>& s1) {
  if constexpr (ACT == kSilu) {  // act_grad's dh (s + h (1 - s)), two elements per instruction
    const uint64_t sg = f2(s0.s, s1.s);
    const uint64_t f = fma2(f2(s0.hr, s1.hr), sub2(f2(1.0f, 1.0f), sg), sg);
    const uint64_t d = mul2(f2(dh0, dh1), f);
    return Pack<T>::pack(f2_lo(d), f2_hi(d));
  } else if constexpr (ACT == kSigmoid) {  // (dh h) round(1 - h)
    const uint64_t hr = f2(s0.hr, s1.hr);
    const uint64_t om = sub2(f2(1.0f, 1.0f), hr);
    const uint64_t d = mul2(mul2(f2(dh0, dh1), hr), f2(Pack<T>::round(f2_lo(om)), Pack<T>::round(f2_hi(om))));
    return Pack<T>::pack(f2_lo(d), f2_hi(d));
  } else if constexpr (ACT == kLeakyRelu) {
    const uint64_t d = mul2(f2(dh0, dh1), f2(s0.pos ? 1.0f : 0.01f, s1.pos ? 1.0f : 0.01f));
    return Pack<T>::pack(f2_lo(d), f2_hi(d));
  } else {
    return Pack<T>::pack(act_grad<T, ACT>(dh0, s0), act_grad<T, ACT>(dh1, s1));
  }
}

// Packs 2*N fp32 values (activated) into N 16-bit pairs.
template <typename T, int ACT, int N>
__device__ __forceinline__ void act_pack(const uint32_t* v, uint32_t* p) {
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const float z0 = __uint_as_float(v[2 * i]), z1 = __uint_as_float(v[2 * i + 1]);
    if constexpr (ACT == kSilu) {  // act_fwd's u tanh(u) + u, two elements per instruction
      const uint64_t u = mul2(f2(0.5f, 0.5f), f2(z0, z1));
      const uint64_t h = fma2(u, f2(tanh_approx(f2_lo(u)), tanh_approx(f2_hi(u))), u);
      p[i] = Pack<T>::pack(f2_lo(h), f2_hi(h));
    } else if constexpr (ACT == kSigmoid) {
      const uint64_t half = f2(0.5f, 0.5f);
      const uint64_t u = mul2(half, f2(z0, z1));
      const uint64_t h = fma2(half, f2(tanh_approx(f2_lo(u)), tanh_approx(f2_hi(u))), half);
      p[i] = Pack<T>::pack(f2_lo(h), f2_hi(h));
    } else if constexpr (ACT == kLeakyRelu) {
      const uint64_t m = mul2(f2(0.01f, 0.01f), f2(z0, z1));
      p[i] = Pack<T>::pack(fmaxf(z0, f2_lo(m)), fmaxf(z1, f2_hi(m)));
    } else {
      p[i] = Pack<T>::pack(z0, z1);
    }
  }
}

// Packs 2*N fp32 values unchanged.
template <typename T, int N>
__device__ __forceinline__ void plain_pack(const uint32_t* v, uint32_t* p) {
#pragma unroll
  for (int i = 0; i < N; ++i) p[i] = Pack<T>::pack(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
}

}  // namespace fmlp
