/*
 * zero1_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the per-element arithmetic of HybridAgent's ZeroOneAdamW
 * (hybrid_rl/optimizer.py), used by tests/, __graft_entry__.smoke() and the
 * CPU-baseline leg of bench.py as the checker.  Nothing in the product links or
 * calls this file; the product path is the CUDA library under hybridagent_b200/.
 *
 * The reference computes its update with torch eager ops, one fp32 rounding per
 * op.  Each op's rounding form differs between torch's CPU and CUDA kernels, so
 * every form is selectable through the ORA_* bits below:
 *
 *   optimizer.py:186  mean.mul_(beta1).add_(g, alpha=1-beta1)
 *                     ORA_ADD_FMA:      fma(alpha, g, m*b1)      else  m*b1 + round(alpha*g)
 *   optimizer.py:187  variance.mul_(beta2).addcmul_(g, g, value=1-beta2)
 *                     ORA_ADDCMUL_INNER: fma(value, round(g*g), v*b2)
 *                     ORA_ADDCMUL_LEFT:  fma(round(value*g), g, v*b2)
 *                     neither:           v*b2 + round(round(value*g)*g)
 *   optimizer.py:188  (variance / correction2).sqrt().add_(eps)
 *   optimizer.py:189  mean / correction1
 *                     ORA_DIV_RECIP: x * (float)(1.0 / c), the reciprocal taken in
 *                     double and rounded once     else  x / (float)c
 *   optimizer.py:189  master.addcdiv_(mhat, denom, value=-lr)
 *                     ORA_ADDCDIV_FMA:  fma(value, mhat/denom, master)
 *                     else:             master + round(round(value*mhat)/denom)
 *   optimizer.py:159  grad.mul_(scale) on a bf16/fp16 gradient
 *                     product float(g) * (float)scale rounded back to the dtype;
 *                     ORA_SCALAR_IN_DTYPE (not torch's behaviour on either device,
 *                     kept to show the difference) rounds the scale to the dtype first
 *
 * Both presets were measured against torch 2.11 on 2^20 random elements per op:
 * ORA_TORCH_CPU against the AVX512 CPU kernels, ORA_TORCH_CUDA against the CUDA
 * kernels on a B200 (tests/test_torch_cuda_forms.py repeats that check).  The CPU
 * form's sqrt is correctly rounded while torch's CPU sqrt (MKL VML) can be 1 ulp away,
 * so it matches the reference's CPU denominators to within 1 ulp.
 *
 * Scalars follow optimizer.py:182-185: corrections 1 - beta**t in double (libm
 * pow, as CPython's float ** does), every Python scalar cast to fp32 once.
 * Conversions to bf16/fp16 are round-to-nearest-even; NaN encodings follow
 * the form (torch CPU: 0x7FC0 / 0x7E00, CUDA cvt: 0x7FFF / 0x7FFF).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define ORA_F32 0
#define ORA_BF16 1
#define ORA_F16 2

#define ORA_ADD_FMA 1u
#define ORA_ADDCMUL_INNER 2u
#define ORA_ADDCMUL_LEFT 4u
#define ORA_DIV_RECIP 8u
#define ORA_ADDCDIV_FMA 16u
#define ORA_SCALAR_IN_DTYPE 32u
#define ORA_NAN_CUDA 64u

#define ORA_TORCH_CPU (ORA_ADD_FMA | ORA_ADDCMUL_LEFT)
#define ORA_TORCH_CUDA (ORA_ADD_FMA | ORA_ADDCMUL_INNER | ORA_DIV_RECIP | ORA_ADDCDIV_FMA | ORA_NAN_CUDA)

static inline float u32_as_f32(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}
static inline uint32_t f32_as_u32(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

static inline float bf16_to_f32(uint16_t b) { return u32_as_f32((uint32_t)b << 16); }

/* float -> bf16, round to nearest even on the 16 dropped bits. */
static inline uint16_t f32_to_bf16(float f, unsigned form) {
  uint32_t u = f32_as_u32(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (form & ORA_NAN_CUDA) ? 0x7fffu : 0x7fc0u;
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* IEEE binary16 <-> binary32 through the compiler's _Float16 (RNE). */
static inline float f16_to_f32(uint16_t h) {
  _Float16 x;
  memcpy(&x, &h, 2);
  return (float)x;
}
static inline uint16_t f32_to_f16(float f, unsigned form) {
  if (isnan(f)) return (form & ORA_NAN_CUDA) ? 0x7fffu : 0x7e00u;
  _Float16 x = (_Float16)f;
  uint16_t h;
  memcpy(&h, &x, 2);
  return h;
}

static inline float load_as_f32(int dtype, const void* p, int64_t i) {
  switch (dtype) {
    case ORA_BF16: return bf16_to_f32(((const uint16_t*)p)[i]);
    case ORA_F16: return f16_to_f32(((const uint16_t*)p)[i]);
    default: return ((const float*)p)[i];
  }
}

static inline void store_from_f32(int dtype, void* p, int64_t i, float x, unsigned form) {
  switch (dtype) {
    case ORA_BF16: ((uint16_t*)p)[i] = f32_to_bf16(x, form); break;
    case ORA_F16: ((uint16_t*)p)[i] = f32_to_f16(x, form); break;
    default: ((float*)p)[i] = x; break;
  }
}

/* The fp32 multiplier torch applies for `tensor.mul_(scale)` (optimizer.py:159). */
float ora_clip_multiplier(int dtype, unsigned form, double scale) {
  float s = (float)scale;
  if ((form & ORA_SCALAR_IN_DTYPE) && dtype == ORA_BF16) s = bf16_to_f32(f32_to_bf16(s, form));
  if ((form & ORA_SCALAR_IN_DTYPE) && dtype == ORA_F16) s = f16_to_f32(f32_to_f16(s, form));
  return s;
}

/* grad.mul_(scale) in the gradient's own dtype, in place (optimizer.py:155-159). */
void ora_clip_inplace(int dtype, unsigned form, int64_t n, void* grad, double scale) {
  const float s = ora_clip_multiplier(dtype, form, scale);
  for (int64_t i = 0; i < n; ++i) store_from_f32(dtype, grad, i, load_as_f32(dtype, grad, i) * s, form);
}

/* Sum of squares of one gradient tensor, float(g)**2 accumulated in double
 * (optimizer.py:151 sums the same fp32 squares in fp32, in torch's order). */
double ora_sumsq(int dtype, int64_t n, const void* grad) {
  double acc = 0.0;
  for (int64_t i = 0; i < n; ++i) {
    const float g = load_as_f32(dtype, grad, i);
    acc += (double)(g * g);
  }
  return acc;
}

/* Fp32 constants of one tensor's update (optimizer.py:180-189). */
typedef struct {
  float decay;   /* (float)(1 - lr*wd) */
  float b1, a1;  /* (float)beta1, (float)(1 - beta1) */
  float b2, a2;  /* (float)beta2, (float)(1 - beta2) */
  float c1, c2;  /* (float)correction */
  float rc1, rc2;/* (float)(1.0 / correction) */
  float eps;     /* (float)eps */
  float neg_lr;  /* (float)(-lr) */
  int use_decay; /* `if self.weight_decay:` */
} ora_consts;

static ora_consts make_consts(double lr, double beta1, double beta2, double eps, double wd, int64_t step) {
  ora_consts k;
  const double c1 = 1.0 - pow(beta1, (double)step);
  const double c2 = 1.0 - pow(beta2, (double)step);
  k.decay = (float)(1.0 - lr * wd);
  k.use_decay = wd != 0.0;
  k.b1 = (float)beta1;
  k.a1 = (float)(1.0 - beta1);
  k.b2 = (float)beta2;
  k.a2 = (float)(1.0 - beta2);
  k.c1 = (float)c1;
  k.c2 = (float)c2;
  k.rc1 = (float)(1.0 / c1);
  k.rc2 = (float)(1.0 / c2);
  k.eps = (float)eps;
  k.neg_lr = (float)(-lr);
  return k;
}

/* Update of one element; g is the (already clipped) gradient widened to fp32. */
static inline void adamw_element(const ora_consts* k, unsigned form, float g, float* master, float* m, float* v) {
  float t; /* one torch op's rounded result; the file is built with -ffp-contract=off */
  float ms = *master;
  if (k->use_decay) ms = ms * k->decay;
  float mb = *m * k->b1;
  float mm;
  if (form & ORA_ADD_FMA) {
    mm = fmaf(k->a1, g, mb);
  } else {
    t = k->a1 * g;
    mm = mb + t;
  }
  float vb = *v * k->b2;
  float vv;
  if (form & ORA_ADDCMUL_INNER) {
    t = g * g;
    vv = fmaf(k->a2, t, vb);
  } else if (form & ORA_ADDCMUL_LEFT) {
    t = k->a2 * g;
    vv = fmaf(t, g, vb);
  } else {
    t = k->a2 * g;
    t = t * g;
    vv = vb + t;
  }
  float q = (form & ORA_DIV_RECIP) ? vv * k->rc2 : vv / k->c2;
  float den = sqrtf(q) + k->eps;
  float mh = (form & ORA_DIV_RECIP) ? mm * k->rc1 : mm / k->c1;
  if (form & ORA_ADDCDIV_FMA) {
    t = mh / den;
    ms = fmaf(k->neg_lr, t, ms);
  } else {
    t = k->neg_lr * mh;
    t = t / den;
    ms = ms + t;
  }
  *master = ms;
  *m = mm;
  *v = vv;
}

/* One owned tensor's step (optimizer.py:176-191).  param_dtype < 0 means the
 * master is the parameter itself (fp32 parameter, optimizer.py:71-73). */
void ora_adamw_tensor(unsigned form, int grad_dtype, int param_dtype, int64_t n, const void* grad, float* master,
                      float* exp_avg, float* exp_avg_sq, void* param, double lr, double beta1, double beta2,
                      double eps, double weight_decay, int64_t step) {
  const ora_consts k = make_consts(lr, beta1, beta2, eps, weight_decay, step);
  for (int64_t i = 0; i < n; ++i) {
    const float g = load_as_f32(grad_dtype, grad, i);
    adamw_element(&k, form, g, master + i, exp_avg + i, exp_avg_sq + i);
    if (param_dtype >= 0) store_from_f32(param_dtype, param, i, master[i], form);
  }
}

/* Same update with the clip folded in: g = dtype(float(g) * multiplier), as the
 * reference's in-place clip followed by .float() produces. */
void ora_adamw_tensor_clipped(unsigned form, int grad_dtype, int param_dtype, int64_t n, const void* grad,
                              float* master, float* exp_avg, float* exp_avg_sq, void* param, double lr,
                              double beta1, double beta2, double eps, double weight_decay, int64_t step,
                              int clip, double scale) {
  const ora_consts k = make_consts(lr, beta1, beta2, eps, weight_decay, step);
  const float s = ora_clip_multiplier(grad_dtype, form, scale);
  for (int64_t i = 0; i < n; ++i) {
    float g = load_as_f32(grad_dtype, grad, i);
    if (clip) {
      g = g * s;
      if (grad_dtype == ORA_BF16) g = bf16_to_f32(f32_to_bf16(g, form));
      if (grad_dtype == ORA_F16) g = f16_to_f32(f32_to_f16(g, form));
    }
    adamw_element(&k, form, g, master + i, exp_avg + i, exp_avg_sq + i);
    if (param_dtype >= 0) store_from_f32(param_dtype, param, i, master[i], form);
  }
}

/* Elementwise conversions exposed for tests of the bf16 / fp16 copies. */
void ora_f32_to_bf16(unsigned form, int64_t n, const float* x, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = f32_to_bf16(x[i], form);
}
void ora_f32_to_f16(unsigned form, int64_t n, const float* x, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = f32_to_f16(x[i], form);
}

/* Sum of W ranks' bf16 gradients the way a reduction that rounds to bf16 after
 * every addition does it, ranks added in order 0..W-1 (optimizer.py:136).
 * For W = 2 every reduction algorithm gives this result. */
void ora_bf16_rank_sum(int64_t n, int world, const uint16_t* const* ranks, uint16_t* out) {
  for (int64_t i = 0; i < n; ++i) {
    float acc = bf16_to_f32(ranks[0][i]);
    for (int r = 1; r < world; ++r) acc = bf16_to_f32(f32_to_bf16(acc + bf16_to_f32(ranks[r][i]), ORA_TORCH_CPU));
    out[i] = f32_to_bf16(acc, ORA_TORCH_CPU);
  }
}

int ora_form_torch_cpu(void) { return (int)ORA_TORCH_CPU; }
int ora_form_torch_cuda(void) { return (int)ORA_TORCH_CUDA; }
