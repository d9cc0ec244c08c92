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
    return z * sigmoid_fast(z);
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

// Packs 2*N fp32 values (activated) into N 16-bit pairs.
template <typename T, int ACT, int N>
__device__ __forceinline__ void act_pack(const uint32_t* v, uint32_t* p) {
#pragma unroll
  for (int i = 0; i < N; ++i)
    p[i] = Pack<T>::pack(act_fwd<T, ACT>(__uint_as_float(v[2 * i])), act_fwd<T, ACT>(__uint_as_float(v[2 * i + 1])));
}

// Packs 2*N fp32 values unchanged.
template <typename T, int N>
__device__ __forceinline__ void plain_pack(const uint32_t* v, uint32_t* p) {
#pragma unroll
  for (int i = 0; i < N; ++i) p[i] = Pack<T>::pack(__uint_as_float(v[2 * i]), __uint_as_float(v[2 * i + 1]));
}

}  // namespace fmlp
