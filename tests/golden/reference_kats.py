"""Known-answer vectors of LightShip's own tests for the dense-contraction path.

Transcribed (inputs, expected outputs and tolerances) from the reference's Rust test
sources, which cannot be run here (no Rust toolchain).  Paths are relative to the
reference project root; ``core/`` = ``lightship-core/src/``, ``tests/`` =
``lightship-core/tests/``.  Both the CPU oracle and the CUDA backend are checked against
these vectors.
"""

# core/cpu/quantized_ops.rs:121-133 -- quantized_gemm_int8, A 2x3 and B 3x2 (NN), i32
QGEMM_A = [1, 2, 3, 4, 5, 6]
QGEMM_B = [1, 2, 3, 4, 5, 6]
QGEMM_MNK = (2, 2, 3)
QGEMM_C = [22, 28, 49, 64]

# core/cpu/quantized_ops.rs:135-146 -- dequantize(i32 * 0.5), exact equality
DEQUANT_IN = [1, 2, 4]
DEQUANT_SCALE = 0.5
DEQUANT_OUT = [0.5, 1.0, 2.0]

# core/cpu/quantized_ops.rs:148-159 -- quantize_sym(x / 0.5), exact equality
QSYM_IN = [0.5, 1.0, 2.0]
QSYM_SCALE = 0.5
QSYM_OUT = [1, 2, 4]

# core/platform/simd.rs:2207-2220 -- gemm_simd 2x3 * 3x2, exact equality
GEMM_A = [1.0, 2.0, 3.0, 4.0, 5.0, 6.0]
GEMM_B = [1.0, 2.0, 3.0, 4.0, 5.0, 6.0]
GEMM_MNK = (2, 2, 3)
GEMM_C = [22.0, 28.0, 49.0, 64.0]
# core/platform/simd.rs:2247-2260 -- C = A*B + C with C0 = [10,20,30,40]
GEMM_C0 = [10.0, 20.0, 30.0, 40.0]
GEMM_C_ACC = [32.0, 48.0, 79.0, 104.0]

# core/platform/simd.rs:2222-2245 -- ramp a[i]=0.01*i, b[i]=0.02*i, 128x256x128; C entries
# (0,0), (0,1), (63,128) within 0.1 of a sequential f32 sum
GEMM_RAMP_LARGE = dict(m=128, n=256, k=128, a_step=0.01, b_step=0.02,
                       points=[(0, 0), (0, 1), (63, 128)], abs_tol=0.1)
# core/platform/simd.rs:2263-2295 -- blocked vs scalar, a=b=0.1*i, relative error < 1e-3
GEMM_BLOCK_ALIGNMENT = dict(cases=[(3, 5, 7), (17, 23, 11), (64, 64, 64), (65, 63, 67)],
                            step=0.1, rel_tol=1e-3)
# core/platform/simd.rs:2297-2315 -- 256^3 ramp, C[100,100] within |e|*1e-3 + 1
GEMM_RAMP_256 = dict(m=256, n=256, k=256, a_step=0.01, b_step=0.02, point=(100, 100))

# core/platform/simd.rs:2164-2182 -- relu / relu6
ACT_IN = [-3.0, -1.0, 0.0, 1.0, 2.0, 5.0, 7.0, 8.0]
RELU_OUT = [0.0, 0.0, 0.0, 1.0, 2.0, 5.0, 7.0, 8.0]
RELU6_OUT = [0.0, 0.0, 0.0, 1.0, 2.0, 5.0, 6.0, 6.0]

# core/operator/silu.rs:162-174 -- SiLU(0)=0 (1e-4), SiLU(1)=0.731, SiLU(-1)=-0.269 (1e-3);
# silu.rs:207-224 -- SiLU(100) within 1 of 100, |SiLU(-100)| < 1e-3
SILU_POINTS = [(0.0, 0.0, 1e-4), (1.0, 0.731, 1e-3), (-1.0, -0.269, 1e-3),
               (100.0, 100.0, 1.0), (-100.0, 0.0, 1e-3)]

# tests/cpu_backend_test.rs:599-662 -- MatMul [2,3] x [3,2], tolerance 1e-3
MATMUL_A = [1.0, 2.0, 3.0, 4.0, 5.0, 6.0]
MATMUL_B = [7.0, 8.0, 9.0, 10.0, 11.0, 12.0]
MATMUL_C = [58.0, 64.0, 139.0, 154.0]
# tests/cpu_backend_test.rs:927-993 -- 32x64 * 64x32 of ones -> 64 everywhere (1e-3)
MATMUL_ONES = dict(m=32, k=64, n=32, value=64.0)

# tests/cpu_backend_test.rs:862-925 -- FullyConnected x=[1,2,3,4], W rows of 1,2,3
FC_X = [1.0, 2.0, 3.0, 4.0]
FC_W = [1.0] * 4 + [2.0] * 4 + [3.0] * 4
FC_Y = [10.0, 20.0, 30.0]

# tests/cpu_backend_test.rs:753-811 and core/operator/convolution.rs:325-376 --
# 1x1x4x4 ones conv 1x1x3x3 ones, s1 p0 -> [1,1,2,2] of 9 (1e-5 / 1e-3)
CONV_ONES = dict(x_shape=(1, 1, 4, 4), w_shape=(1, 1, 3, 3), y_shape=(1, 1, 2, 2), value=9.0)
# tests/cpu_backend_test.rs:995-1069 -- batch b filled with (b+1) -> 9*(b+1)
CONV_BATCHED = dict(x_shape=(4, 1, 4, 4), w_shape=(1, 1, 3, 3), y_shape=(4, 1, 2, 2))
# core/operator/convolution.rs:378-409 -- 2x2 stride-2 conv on 4x4 -> [1,1,2,2]
CONV_STRIDE2 = dict(x_shape=(1, 1, 4, 4), w_shape=(1, 1, 2, 2), stride=2, y_shape=(1, 1, 2, 2))
# core/operator/convolution.rs:411-447 -- groups=2, channels filled 1,2,3,4, 1x1 ones filter
CONV_GROUPS = dict(x_shape=(1, 4, 2, 2), w_shape=(4, 2, 1, 1), groups=2, y_shape=(1, 4, 2, 2),
                   channel_values=[1.0, 2.0, 3.0, 4.0])
# core/operator/convolution.rs:305-322 -- output_shape 32x32, 3x3, s1, p1 -> 32x32
CONV_OUT_SHAPE = dict(in_hw=32, k=3, stride=1, pad=1, dil=1, out=32)
# tests/onnx_integration_test.rs:117-220 -- conv_relu fixture shapes: X 1x3x32x32,
# W 16x3x3x3, B 16 -> 1x16x30x30
ONNX_CONV_RELU = dict(x_shape=(1, 3, 32, 32), w_shape=(16, 3, 3, 3), y_shape=(1, 16, 30, 30))

# tests/cpu_backend_test.rs:813-860 -- BatchNorm defaults on 4.0 -> 4.0 (1e-3)
BN_DEFAULTS = dict(shape=(1, 2, 2, 2), value=4.0, tol=1e-3)
# core/operator/batchnorm.rs:447-475 -- mean 2, var 1: x - 2
BN_NONZERO_MEAN = dict(x=[0.0, 1.0, 2.0, 3.0], mean=[2.0], var=[1.0], gamma=[1.0], beta=[0.0],
                       y=[-2.0, -1.0, 0.0, 1.0])
# core/operator/batchnorm.rs:479-507 -- gamma 2, beta 1: 2x + 1
BN_GAMMA_BETA = dict(x=[0.0, 1.0, 2.0, 3.0], mean=[0.0], var=[1.0], gamma=[2.0], beta=[1.0],
                     y=[1.0, 3.0, 5.0, 7.0])
# core/operator/batchnorm.rs:551-586 -- two channels
BN_MULTI = dict(x=[0.0, 1.0, 0.0, 1.0], mean=[0.0, 1.0], var=[1.0, 4.0], gamma=[1.0, 0.5],
                beta=[0.0, 1.0], y=[0.0, 1.0, 0.75, 1.0], shape=(1, 2, 2))

# tests/quantization_test.rs:85-99 -- find_scale_zp on [-1,-0.5,0,0.5,1]
FSZ_DATA = [-1.0, -0.5, 0.0, 0.5, 1.0]
# tests/quantization_test.rs:101-111 -- 0.5 at scale 0.01, zp 0 round-trips within 0.1
ROUNDTRIP = dict(value=0.5, scale=0.01, zp=0, tol=0.1)
