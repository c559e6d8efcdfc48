// CPU restatements of the two ncnn built-in layers the reference's hot-path
// layers instantiate, so that the reference sources link into the oracle.
// TEST INFRASTRUCTURE ONLY (never linked into the shipped library).
//
// ncnn itself (Tencent/ncnn @ 3b7bdba7fc8aea8fd46779533eee027df77c639d,
// pinned in the reference's CMakeLists.txt:10) is not available here, so the
// published behaviour of its layers is restated:
//
//   SDPA   (configured in adaptive_window_attention.cpp:847-861: param 5
//           attn_mask=0, 6 scale=0 -> 1/sqrt(head_dim), 7 kv_cache=0)
//          out[h][i] = sum_j softmax_j(scale * q[h][i] . k[h][j]) v[h][j],
//          fp32, max-subtracted softmax over all keys, no mask.
//
//   Gemm   (configured in shared_linear.cpp:27-59: alpha=1, beta=1, transA=0,
//           transB=1, constantB=1, constantC=1, N=num_output, K=num_input,
//           broadcast_type_C 4 = per-output row vector, -1 = no C)
//          out[m][n] = sum_k A[m][k] * B[n][k] + C[n], fp32.
//
//   Convolution (configured in decomposed_conv3d.cpp:480-497: 0 num_output,
//           1/11 kernel w/h, 2/12 dilation, 3/13 stride, 4/15/14/16 pad
//           left/right/top/bottom, 5 bias_term, 6 weight_data_size; weights
//           [num_output][num_input][kernel_h][kernel_w])
//          out[p][y][x] = bias[p] + sum_{q, ky, kx} w[p][q][ky][kx] *
//                         in[q][y*sh + ky*dh - pt][x*sw + kx*dw - pl]
//          with zeros outside the input, fp32, summed in (q, ky, kx) order.
//
//   MultiHeadAttention (configured in vae_chunked_mha.cpp:144-162 with one
//           input blob [tokens][qdim]: 0 embed_dim, 1 num_heads, 2
//           weight_data_size, 3 kdim, 4 vdim, 5 attn_mask = 0, 6 scale;
//           weights q, k, v [embed_dim][in] + bias, out [qdim][embed_dim] +
//           bias)
//          q/k/v = x W^T + b; per head softmax(scale q k^T) v (fp32,
//          max-subtracted, normalised after the sum); out = o Wout^T + b.
//
// All loops parallelise with OpenMP over independent outputs, so results do
// not depend on the thread count.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "layer.h"

namespace ncnn {

namespace {

class ShimSDPA : public Layer
{
public:
    ShimSDPA() : attn_mask(0), scale(0.f), kv_cache(0)
    {
        one_blob_only = false;
        support_inplace = false;
    }

    virtual int load_param(const ParamDict& pd)
    {
        attn_mask = pd.get(5, 0);
        scale = pd.get(6, 0.f);
        kv_cache = pd.get(7, 0);
        return (attn_mask != 0 || kv_cache != 0) ? -1 : 0;
    }

    virtual int forward(const std::vector<Mat>& bottom, std::vector<Mat>& top, const Option& opt) const
    {
        if (bottom.size() != 3 || top.size() != 1) return -1;
        const Mat& q = bottom[0];
        const Mat& k = bottom[1];
        const Mat& v = bottom[2];
        const int d = q.w;
        const int sq = q.h;
        const int heads = q.c;
        const int sk = k.h;
        const int dv = v.w;
        if (k.w != d || k.c != heads || v.h != sk || v.c != heads) return -1;
        const float s = scale == 0.f ? 1.f / std::sqrt((float)d) : scale;

        Mat& out = top[0];
        out.create(dv, sq, heads, 4u, opt.blob_allocator);
        if (out.empty()) return -100;

#pragma omp parallel for schedule(dynamic, 1) collapse(2)
        for (int h = 0; h < heads; h++)
        {
            for (int i = 0; i < sq; i++)
            {
                std::vector<float> logits(sk);
                const float* qi = q.channel(h).row(i);
                float m = -INFINITY;
                for (int j = 0; j < sk; j++)
                {
                    const float* kj = k.channel(h).row(j);
                    float acc = 0.f;
                    for (int t = 0; t < d; t++) acc += qi[t] * kj[t];
                    logits[j] = acc * s;
                    if (logits[j] > m) m = logits[j];
                }
                float sum = 0.f;
                for (int j = 0; j < sk; j++)
                {
                    logits[j] = std::exp(logits[j] - m);
                    sum += logits[j];
                }
                const float inv = 1.f / sum;
                float* oi = out.channel(h).row(i);
                for (int t = 0; t < dv; t++) oi[t] = 0.f;
                for (int j = 0; j < sk; j++)
                {
                    const float p = logits[j] * inv;
                    const float* vj = v.channel(h).row(j);
                    for (int t = 0; t < dv; t++) oi[t] += p * vj[t];
                }
            }
        }
        return 0;
    }

private:
    int attn_mask;
    float scale;
    int kv_cache;
};

class ShimGemm : public Layer
{
public:
    ShimGemm() : alpha(1.f), beta(1.f), transA(0), transB(0), constantB(0), constantC(0), N(0), K(0), bcastC(-1)
    {
        one_blob_only = true;
        support_inplace = false;
    }

    virtual int load_param(const ParamDict& pd)
    {
        alpha = pd.get(0, 1.f);
        beta = pd.get(1, 1.f);
        transA = pd.get(2, 0);
        transB = pd.get(3, 0);
        constantB = pd.get(5, 0);
        constantC = pd.get(6, 0);
        N = pd.get(8, 0);
        K = pd.get(9, 0);
        bcastC = pd.get(10, 0);
        // Only the configuration SharedLinear uses is restated.
        if (transA != 0 || transB != 1 || constantB != 1 || constantC != 1 || N <= 0 || K <= 0) return -1;
        if (bcastC != 4 && bcastC != -1) return -1;
        return 0;
    }

    virtual int load_model(const ModelBin& mb)
    {
        B = mb.load(K * N, 0);
        if (B.empty()) return -100;
        if (bcastC == 4)
        {
            C = mb.load(N, 0);
            if (C.empty()) return -100;
        }
        return 0;
    }

    virtual int forward(const Mat& A, Mat& out, const Option& opt) const
    {
        if (A.dims != 2 || A.w != K) return -1;
        const int M = A.h;
        out.create(N, M, 4u, opt.blob_allocator);
        if (out.empty()) return -100;
        const float* bdata = (const float*)B.data;
        const float* cdata = bcastC == 4 ? (const float*)C.data : 0;

        // 4x4 register tiles of dot products over contiguous K.
#pragma omp parallel for schedule(dynamic, 1)
        for (int m0 = 0; m0 < M; m0 += 4)
        {
            const int mr = M - m0 < 4 ? M - m0 : 4;
            for (int n0 = 0; n0 < N; n0 += 4)
            {
                const int nr = N - n0 < 4 ? N - n0 : 4;
                float acc[4][4] = {{0.f}};
                const float* a[4];
                const float* b[4];
                for (int r = 0; r < 4; r++)
                {
                    a[r] = A.row(m0 + (r < mr ? r : 0));
                    b[r] = bdata + (size_t)(n0 + (r < nr ? r : 0)) * K;
                }
                for (int r = 0; r < 4; r++)
                {
                    for (int c = 0; c < 4; c++)
                    {
                        float s = 0.f;
                        const float* ar = a[r];
                        const float* bc = b[c];
#pragma omp simd reduction(+ : s)
                        for (int t = 0; t < K; t++) s += ar[t] * bc[t];
                        acc[r][c] = s;
                    }
                }
                for (int r = 0; r < mr; r++)
                {
                    float* o = out.row(m0 + r);
                    for (int c = 0; c < nr; c++)
                        o[n0 + c] = alpha * acc[r][c] + (cdata ? beta * cdata[n0 + c] : 0.f);
                }
            }
        }
        return 0;
    }

private:
    float alpha;
    float beta;
    int transA;
    int transB;
    int constantB;
    int constantC;
    int N;
    int K;
    int bcastC;
    Mat B;
    Mat C;
};

} // namespace

namespace {

class ShimConvolution : public Layer
{
public:
    ShimConvolution()
        : num_output(0), kernel_w(0), kernel_h(0), dilation_w(1), dilation_h(1), stride_w(1), stride_h(1),
          pad_left(0), pad_right(0), pad_top(0), pad_bottom(0), bias_term(0), weight_data_size(0)
    {
        one_blob_only = true;
        support_inplace = false;
    }

    virtual int load_param(const ParamDict& pd)
    {
        num_output = pd.get(0, 0);
        kernel_w = pd.get(1, 0);
        kernel_h = pd.get(11, kernel_w);
        dilation_w = pd.get(2, 1);
        dilation_h = pd.get(12, dilation_w);
        stride_w = pd.get(3, 1);
        stride_h = pd.get(13, stride_w);
        pad_left = pd.get(4, 0);
        pad_right = pd.get(15, pad_left);
        pad_top = pd.get(14, pad_left);
        pad_bottom = pd.get(16, pad_top);
        bias_term = pd.get(5, 0);
        weight_data_size = pd.get(6, 0);
        // negative pads are ncnn's "same" modes, not used by the reference layer
        if (num_output <= 0 || kernel_w <= 0 || kernel_h <= 0 || pad_left < 0 || pad_right < 0 || pad_top < 0 ||
            pad_bottom < 0)
            return -1;
        return 0;
    }

    virtual int load_model(const ModelBin& mb)
    {
        weight_data = mb.load(weight_data_size, 0);
        if (weight_data.empty()) return -100;
        if (bias_term)
        {
            bias_data = mb.load(num_output, 1);
            if (bias_data.empty()) return -100;
        }
        return 0;
    }

    virtual int forward(const Mat& bottom, Mat& top, const Option& opt) const
    {
        const int w = bottom.w, h = bottom.h, inch = bottom.c;
        if (inch <= 0 || weight_data_size != num_output * inch * kernel_w * kernel_h) return -1;
        const int ew = dilation_w * (kernel_w - 1) + 1, eh = dilation_h * (kernel_h - 1) + 1;
        const int outw = (w + pad_left + pad_right - ew) / stride_w + 1;
        const int outh = (h + pad_top + pad_bottom - eh) / stride_h + 1;
        if (outw <= 0 || outh <= 0) return -1;
        top.create(outw, outh, num_output, 4u, opt.blob_allocator);
        if (top.empty()) return -100;
        const float* wt = weight_data;
#pragma omp parallel for schedule(static)
        for (int p = 0; p < num_output; p++)
        {
            float* out = top.channel(p);
            for (int y = 0; y < outh; y++)
                for (int x = 0; x < outw; x++)
                {
                    float sum = bias_term ? ((const float*)bias_data)[p] : 0.f;
                    for (int q = 0; q < inch; q++)
                    {
                        const float* in = bottom.channel(q);
                        const float* kq = wt + ((size_t)p * inch + q) * kernel_h * kernel_w;
                        for (int ky = 0; ky < kernel_h; ky++)
                        {
                            const int iy = y * stride_h + ky * dilation_h - pad_top;
                            if (iy < 0 || iy >= h) continue;
                            for (int kx = 0; kx < kernel_w; kx++)
                            {
                                const int ix = x * stride_w + kx * dilation_w - pad_left;
                                if (ix < 0 || ix >= w) continue;
                                sum += in[(size_t)iy * w + ix] * kq[ky * kernel_w + kx];
                            }
                        }
                    }
                    out[(size_t)y * outw + x] = sum;
                }
        }
        return 0;
    }

private:
    int num_output, kernel_w, kernel_h, dilation_w, dilation_h, stride_w, stride_h;
    int pad_left, pad_right, pad_top, pad_bottom, bias_term, weight_data_size;
    Mat weight_data, bias_data;
};

// y[t][o] = b[o] + sum_i x[t][i] w[o][i], fp32 in i order
void shim_linear(const float* x, int tokens, int in, const float* w, const float* b, int out, float* y)
{
#pragma omp parallel for schedule(static)
    for (int t = 0; t < tokens; t++)
        for (int o = 0; o < out; o++)
        {
            float sum = b[o];
            const float* xr = x + (size_t)t * in;
            const float* wr = w + (size_t)o * in;
            for (int i = 0; i < in; i++) sum += xr[i] * wr[i];
            y[(size_t)t * out + o] = sum;
        }
}

class ShimMultiHeadAttention : public Layer
{
public:
    ShimMultiHeadAttention() : embed_dim(0), num_heads(1), weight_data_size(0), kdim(0), vdim(0), attn_mask(0), scale(1.f)
    {
        one_blob_only = false;
        support_inplace = false;
    }

    virtual int load_param(const ParamDict& pd)
    {
        embed_dim = pd.get(0, 0);
        num_heads = pd.get(1, 1);
        weight_data_size = pd.get(2, 0);
        kdim = pd.get(3, embed_dim);
        vdim = pd.get(4, embed_dim);
        attn_mask = pd.get(5, 0);
        scale = pd.get(6, 1.f);
        if (embed_dim <= 0 || num_heads <= 0 || embed_dim % num_heads || attn_mask != 0) return -1;
        return 0;
    }

    virtual int load_model(const ModelBin& mb)
    {
        const int qdim = weight_data_size / embed_dim;
        for (int i = 0; i < 8; i++)
        {
            const int n = i == 0 ? embed_dim * qdim : i == 2 ? embed_dim * kdim : i == 4 ? embed_dim * vdim
                          : i == 6 ? qdim * embed_dim : (i == 7 ? qdim : embed_dim);
            w[i] = mb.load(n, i % 2 ? 1 : 0);
            if (w[i].empty()) return -100;
        }
        return 0;
    }

    virtual int forward(const std::vector<Mat>& bottom, std::vector<Mat>& top, const Option& opt) const
    {
        // one input blob: self-attention (q, k and v read it)
        if (bottom.size() != 1 || top.size() != 1) return -1;
        const Mat& x = bottom[0];
        const int qdim = weight_data_size / embed_dim;
        const int T = x.h;
        if (x.w != qdim || kdim != qdim || vdim != qdim) return -1;
        const int E = embed_dim, hd = E / num_heads;
        std::vector<float> q((size_t)T * E), k((size_t)T * E), v((size_t)T * E), o((size_t)T * E);
        shim_linear((const float*)x.data, T, qdim, w[0], w[1], E, q.data());
        shim_linear((const float*)x.data, T, kdim, w[2], w[3], E, k.data());
        shim_linear((const float*)x.data, T, vdim, w[4], w[5], E, v.data());
#pragma omp parallel for schedule(static)
        for (int t = 0; t < T; t++)
        {
            std::vector<float> s((size_t)T);
            for (int h = 0; h < num_heads; h++)
            {
                const float* qr = q.data() + (size_t)t * E + h * hd;
                float m = -INFINITY;
                for (int j = 0; j < T; j++)
                {
                    const float* kr = k.data() + (size_t)j * E + h * hd;
                    float d = 0.f;
                    for (int i = 0; i < hd; i++) d += qr[i] * kr[i];
                    s[j] = d * scale;
                    m = std::max(m, s[j]);
                }
                float sum = 0.f;
                for (int j = 0; j < T; j++)
                {
                    s[j] = std::exp(s[j] - m);
                    sum += s[j];
                }
                float* orow = o.data() + (size_t)t * E + h * hd;
                for (int i = 0; i < hd; i++) orow[i] = 0.f;
                for (int j = 0; j < T; j++)
                {
                    const float p = s[j] / sum;
                    const float* vr = v.data() + (size_t)j * E + h * hd;
                    for (int i = 0; i < hd; i++) orow[i] += p * vr[i];
                }
            }
        }
        Mat& y = top[0];
        y.create(qdim, T, 4u, opt.blob_allocator);
        if (y.empty()) return -100;
        shim_linear(o.data(), T, E, w[6], w[7], qdim, (float*)y.data);
        return 0;
    }

private:
    int embed_dim, num_heads, weight_data_size, kdim, vdim, attn_mask;
    float scale;
    Mat w[8];
};

} // namespace

Layer* create_layer(const char* type)
{
    const std::string t(type ? type : "");
    if (t == "SDPA") return new ShimSDPA;
    if (t == "Gemm") return new ShimGemm;
    if (t == "Convolution") return new ShimConvolution;
    if (t == "MultiHeadAttention") return new ShimMultiHeadAttention;
    return 0;
}

Layer* create_layer_cpu(const char* type)
{
    return create_layer(type);
}

} // namespace ncnn
