// Element-wise task operators for sm_100a.
//
//   silu          y = x * sigmoid(x)              tasks/silu/reference.py:105-108
//   swiglu        y = gate * sigmoid(gate) * up   tasks/swiglu/reference.py:109-113
//   relu          y = max(x, 0), NaN propagates   tasks/relu/reference.py (reference(): torch.relu)
//   sigmoid       y = 1 / (1 + exp(-x))           tasks/sigmoid/reference.py (reference(): torch.sigmoid)
//   sigmoid_shift y = sigmoid(x) + 1              tasks/sigmoid_shift/reference.py
//   lion          c = b1*m + (1-b1)*g; p' = p*(1 - lr*wd) - lr*sign(c); m' = b2*m + (1-b2)*g
//                                                 tasks/lion/reference.py (reference())
//
// HBM-bound (2 to 5 streams of 16-bit elements, a handful of flops each).  A grid-stride loop of
// 16-byte vector loads/stores over one wave of CTAs (SMs x the CTAs that fit on an SM, from the
// occupancy calculator: a second, partial wave of a grid-stride grid leaves most SMs idle at the
// end); the element tail and unaligned bases take a scalar loop.  sigmoid is evaluated in fp32 by sf::sigmoid_nr (one exp and a branch-free
// Newton reciprocal: the IEEE division's second MUFU op made these kernels issue-bound), which maps
// +-Inf and NaN the way the fp64 reference does (sigmoid(-inf) = 0, so silu(-inf) = -inf * 0 = NaN).
#include "sf_common.cuh"

namespace {

enum Act : int { SILU = 0, SWIGLU = 1, RELU = 2, SIGMOID = 3, SIGMOID_SHIFT = 4 };

__device__ __forceinline__ float sigmoidf_(float x) { return sf::sigmoid_nr(x); }

template <int A>
__device__ __forceinline__ float act(float x, float up) {
    if (A == SILU) return x * sigmoidf_(x);
    if (A == SWIGLU) return x * sigmoidf_(x) * up;
    // torch.relu: x > 0 keeps x, NaN stays NaN, everything else (-0 included) is +0.
    if (A == RELU) return x > 0.f ? x : (x != x ? x : 0.f);
    if (A == SIGMOID) return sigmoidf_(x);
    return sigmoidf_(x) + 1.0f;
}

// The same on a pair of values with packed fp32 arithmetic (the vector loop's form: these kernels
// are instruction-issue bound once the sigmoid is in, not HBM bound).
template <int A>
__device__ __forceinline__ float2 act2(float2 x, float2 up) {
    if (A == RELU) return make_float2(act<RELU>(x.x, 0.f), act<RELU>(x.y, 0.f));
    const float2 s = sf::sigmoid2_nr(x);
    if (A == SILU) return sf::f2_mul(x, s);
    if (A == SWIGLU) return sf::f2_mul(sf::f2_mul(x, s), up);
    if (A == SIGMOID) return s;
    return sf::f2_add(s, sf::f2(1.0f));
}

constexpr const char* act_name(int a) {
    return a == SILU ? "silu" : a == SWIGLU ? "swiglu" : a == RELU ? "relu" : a == SIGMOID ? "sigmoid" : "sigmoid_shift";
}

template <typename T, int A>
__device__ __forceinline__ void apply_vec(const sf::Vec8<T>& a, const sf::Vec8<T>& u, T* dst) {
    sf::Vec8<T> o;
    const uint32_t* aw = reinterpret_cast<const uint32_t*>(&a);
    const uint32_t* uw = reinterpret_cast<const uint32_t*>(&u);
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j)
        ow[j] = sf::Pair<T>::from_f2(act2<A>(sf::Pair<T>::to_f2(aw[j]), A == SWIGLU ? sf::Pair<T>::to_f2(uw[j]) : sf::f2(0.f)));
    sf::st_global_v8<T>(dst, o);
}

template <typename T, int A>
__global__ void __launch_bounds__(256) act_kernel(const T* __restrict__ x, const T* __restrict__ up, T* __restrict__ y,
                                                  int64_t n, bool vec) {
    constexpr bool GLU = A == SWIGLU;
    // The sigmoid-based unary operators carry enough arithmetic per element that a thread's load
    // and compute phases no longer overlap across warps; they double-buffer in registers (the next
    // step's two vectors are requested before this step's are computed).  relu and swiglu (two
    // input streams) keep the plain two-vector step, which needs fewer registers.
    constexpr bool PREFETCH = A == SILU || A == SIGMOID || A == SIGMOID_SHIFT;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t done = 0;
    if (vec) {
        const int64_t nv = n >> 3;
        if constexpr (PREFETCH) {
            sf::Vec8<T> a0, a1, u;
            if (tid < nv) a0 = sf::ld_global_nc_v8<T>(x + tid * 8);
            if (tid + stride < nv) a1 = sf::ld_global_nc_v8<T>(x + (tid + stride) * 8);
            for (int64_t i = tid; i < nv; i += 2 * stride) {
                const int64_t j0 = i + 2 * stride, j1 = i + 3 * stride;
                sf::Vec8<T> b0, b1;
                if (j0 < nv) b0 = sf::ld_global_nc_v8<T>(x + j0 * 8);
                if (j1 < nv) b1 = sf::ld_global_nc_v8<T>(x + j1 * 8);
                apply_vec<T, A>(a0, u, y + i * 8);
                if (i + stride < nv) apply_vec<T, A>(a1, u, y + (i + stride) * 8);
                a0 = b0;
                a1 = b1;
            }
        } else {
            int64_t i = tid;
            // relu: two independent vectors per thread and step, so twice the bytes are in flight
            // (swiglu already has two input streams per vector).
            for (; !GLU && i + stride < nv; i += 2 * stride) {
                const sf::Vec8<T> a0 = sf::ld_global_nc_v8<T>(x + i * 8);
                const sf::Vec8<T> a1 = sf::ld_global_nc_v8<T>(x + (i + stride) * 8);
                sf::Vec8<T> u;
                apply_vec<T, A>(a0, u, y + i * 8);
                apply_vec<T, A>(a1, u, y + (i + stride) * 8);
            }
            for (; i < nv; i += stride) {
                sf::Vec8<T> u0;
                if (GLU) u0 = sf::ld_global_nc_v8<T>(up + i * 8);
                apply_vec<T, A>(sf::ld_global_nc_v8<T>(x + i * 8), u0, y + i * 8);
            }
        }
        done = nv * 8;
    }
    for (int64_t i = done + tid; i < n; i += stride) {
        const float f = sf::Dt<T>::to_f(x[i]);
        y[i] = sf::Dt<T>::from_f(act<A>(f, GLU ? sf::Dt<T>::to_f(up[i]) : 0.f));
    }
}

// One wave of grid-stride CTAs: at most SMs x the CTAs of this kernel that fit on an SM.
int64_t grid_for(int64_t work, int resident) {
    int64_t blocks = (work + 255) / 256;
    const int64_t cap_blocks = (int64_t)sf::sm_count() * resident;
    if (blocks > cap_blocks) blocks = cap_blocks;
    return blocks < 1 ? 1 : blocks;
}

template <typename T, int A>
int launch_t(const void* x, const void* up, void* y, int64_t n, int32_t variant, cudaStream_t s, char* err, uint64_t cap) {
    const bool vec = variant != 2 && sf::aligned16(x) && sf::aligned16(y) && (A != SWIGLU || sf::aligned16(up));
    static const int resident = sf::resident_ctas(act_kernel<T, A>, 256, 0);
    const int64_t blocks = grid_for(vec ? (n + 7) / 8 : n, resident);
    act_kernel<T, A><<<(unsigned)blocks, 256, 0, s>>>((const T*)x, (const T*)up, (T*)y, n, vec);
    return sf::check_launch(act_name(A), err, cap);
}

template <int A>
int launch(const void* x, const void* up, void* y, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s, char* err,
           uint64_t cap) {
    const char* name = act_name(A);
    if (n < 0) return sf::fail(SF_EINVAL, err, cap, "%s: negative size", name);
    if (n == 0) return SF_OK;
    if (!x || !y || (A == SWIGLU && !up)) return sf::fail(SF_EINVAL, err, cap, "%s: null tensor pointer", name);
    if (dtype == SF_DTYPE_F16) return launch_t<__half, A>(x, up, y, n, variant, s, err, cap);
    if (dtype == SF_DTYPE_BF16) return launch_t<__nv_bfloat16, A>(x, up, y, n, variant, s, err, cap);
    return sf::fail(SF_EINVAL, err, cap, "%s: dtype %d is not fp16/bf16", name, dtype);
}

// ---- lion ---------------------------------------------------------------------------------------

struct LionCoef {
    float decay;  // 1 - lr * wd
    float lr;
    float b1, c1;  // beta1, 1 - beta1
    float b2, c2;  // beta2, 1 - beta2
};

// torch.sign: +1 / -1 for non-zero values, 0 for +-0 and for NaN (a NaN c only decays p).
__device__ __forceinline__ float sign_f(float c) { return c > 0.f ? 1.f : (c < 0.f ? -1.f : 0.f); }

template <typename T>
__device__ __forceinline__ void lion_one(float p, float g, float m, const LionCoef& k, T& p_out, T& m_out) {
    const float c = fmaf(k.b1, m, k.c1 * g);
    p_out = sf::Dt<T>::from_f(fmaf(-k.lr, sign_f(c), p * k.decay));
    m_out = sf::Dt<T>::from_f(fmaf(k.b2, m, k.c2 * g));
}

template <typename T>
__global__ void __launch_bounds__(256) lion_kernel(const T* __restrict__ p, const T* __restrict__ g, const T* __restrict__ m,
                                                   T* __restrict__ p_out, T* __restrict__ m_out, int64_t n, LionCoef k, bool vec) {
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t done = 0;
    if (vec) {
        const int64_t nv = n >> 3;
        for (int64_t i = tid; i < nv; i += stride) {
            const sf::Vec8<T> pv = sf::ld_global_nc_v8<T>(p + i * 8);
            const sf::Vec8<T> gv = sf::ld_global_nc_v8<T>(g + i * 8);
            const sf::Vec8<T> mv = sf::ld_global_nc_v8<T>(m + i * 8);
            sf::Vec8<T> po, mo;
#pragma unroll
            for (int j = 0; j < 8; ++j)
                lion_one<T>(sf::Dt<T>::to_f(pv.v[j]), sf::Dt<T>::to_f(gv.v[j]), sf::Dt<T>::to_f(mv.v[j]), k, po.v[j], mo.v[j]);
            sf::st_global_v8<T>(p_out + i * 8, po);
            sf::st_global_v8<T>(m_out + i * 8, mo);
        }
        done = nv * 8;
    }
    for (int64_t i = done + tid; i < n; i += stride)
        lion_one<T>(sf::Dt<T>::to_f(p[i]), sf::Dt<T>::to_f(g[i]), sf::Dt<T>::to_f(m[i]), k, p_out[i], m_out[i]);
}

template <typename T>
int lion_t(const void* p, const void* g, const void* m, void* p_out, void* m_out, int64_t n, const LionCoef& k, int32_t variant,
           cudaStream_t s, char* err, uint64_t cap) {
    const bool vec = variant != 2 && sf::aligned16(p) && sf::aligned16(g) && sf::aligned16(m) && sf::aligned16(p_out) &&
                     sf::aligned16(m_out);
    static const int resident = sf::resident_ctas(lion_kernel<T>, 256, 0);
    const int64_t blocks = grid_for(vec ? (n + 7) / 8 : n, resident);
    lion_kernel<T><<<(unsigned)blocks, 256, 0, s>>>((const T*)p, (const T*)g, (const T*)m, (T*)p_out, (T*)m_out, n, k, vec);
    return sf::check_launch("lion launch", err, cap);
}

}  // namespace

int sf_silu_launch(const void* x, void* y, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s, char* err, uint64_t cap) {
    return launch<SILU>(x, nullptr, y, n, dtype, variant, s, err, cap);
}

int sf_swiglu_launch(const void* gate, const void* up, void* y, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s,
                     char* err, uint64_t cap) {
    return launch<SWIGLU>(gate, up, y, n, dtype, variant, s, err, cap);
}

int sf_relu_launch(const void* x, void* y, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s, char* err, uint64_t cap) {
    return launch<RELU>(x, nullptr, y, n, dtype, variant, s, err, cap);
}

int sf_sigmoid_launch(const void* x, void* y, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s, char* err, uint64_t cap) {
    return launch<SIGMOID>(x, nullptr, y, n, dtype, variant, s, err, cap);
}

int sf_sigmoid_shift_launch(const void* x, void* y, int64_t n, int32_t dtype, int32_t variant, cudaStream_t s, char* err,
                            uint64_t cap) {
    return launch<SIGMOID_SHIFT>(x, nullptr, y, n, dtype, variant, s, err, cap);
}

// Attribute domains of tasks/lion/opspec.json: LR > 0, WD >= 0, 0 < BETA1 < 1, 0 < BETA2 < 1.
int sf_lion_launch(const void* p, const void* g, const void* m, void* p_out, void* m_out, int64_t n, double lr, double wd,
                   double beta1, double beta2, int32_t dtype, int32_t variant, cudaStream_t s, char* err, uint64_t cap) {
    if (n < 0) return sf::fail(SF_EINVAL, err, cap, "lion: negative size");
    if (!(lr > 0.0) || !(wd >= 0.0) || !(beta1 > 0.0 && beta1 < 1.0) || !(beta2 > 0.0 && beta2 < 1.0))
        return sf::fail(SF_EINVAL, err, cap, "lion: attributes out of domain (LR > 0, WD >= 0, 0 < BETA1, BETA2 < 1)");
    if (n == 0) return SF_OK;
    if (!p || !g || !m || !p_out || !m_out) return sf::fail(SF_EINVAL, err, cap, "lion: null tensor pointer");
    const LionCoef k{(float)(1.0 - lr * wd), (float)lr, (float)beta1, (float)(1.0 - beta1), (float)beta2, (float)(1.0 - beta2)};
    if (dtype == SF_DTYPE_F16) return lion_t<__half>(p, g, m, p_out, m_out, n, k, variant, s, err, cap);
    if (dtype == SF_DTYPE_BF16) return lion_t<__nv_bfloat16>(p, g, m, p_out, m_out, n, k, variant, s, err, cap);
    return sf::fail(SF_EINVAL, err, cap, "lion: dtype %d is not fp16/bf16", dtype);
}

extern "C" int sf_silu(const void* x, void* y, int64_t n, int32_t dtype, void* stream, char* err, uint64_t cap) {
    return sf_silu_launch(x, y, n, dtype, 0, (cudaStream_t)stream, err, cap);
}

extern "C" int sf_swiglu(const void* gate, const void* up, void* y, int64_t n, int32_t dtype, void* stream, char* err,
                         uint64_t cap) {
    return sf_swiglu_launch(gate, up, y, n, dtype, 0, (cudaStream_t)stream, err, cap);
}

extern "C" int sf_relu(const void* x, void* y, int64_t n, int32_t dtype, void* stream, char* err, uint64_t cap) {
    return sf_relu_launch(x, y, n, dtype, 0, (cudaStream_t)stream, err, cap);
}

extern "C" int sf_sigmoid(const void* x, void* y, int64_t n, int32_t dtype, void* stream, char* err, uint64_t cap) {
    return sf_sigmoid_launch(x, y, n, dtype, 0, (cudaStream_t)stream, err, cap);
}

extern "C" int sf_sigmoid_shift(const void* x, void* y, int64_t n, int32_t dtype, void* stream, char* err, uint64_t cap) {
    return sf_sigmoid_shift_launch(x, y, n, dtype, 0, (cudaStream_t)stream, err, cap);
}

extern "C" int sf_lion(const void* p, const void* g, const void* m, void* p_out, void* m_out, int64_t n, double lr, double wd,
                       double beta1, double beta2, int32_t dtype, void* stream, char* err, uint64_t cap) {
    return sf_lion_launch(p, g, m, p_out, m_out, n, lr, wd, beta1, beta2, dtype, 0, (cudaStream_t)stream, err, cap);
}
