// Clean-room ModelBin subset for compiling the reference's layer sources into
// the CPU oracle.  TEST INFRASTRUCTURE ONLY.
//
// ModelBin::load(w, type) returns the next weight blob of w elements.  Type 1
// means raw fp32 (adaptive_window_attention.cpp:716-738,
// shared_linear.cpp:61-80, decomposed_conv3d.cpp:425-466); type 0 is ncnn's
// tagged form, whose fp32 variant is a zero tag word before the values --
// the oracle's flat float arrays carry the values only, so both types read
// raw fp32 here (vae_chunked_mha.cpp:126-135 asks for type 0).
#ifndef S2_ORACLE_NCNN_SHIM_MODELBIN_H
#define S2_ORACLE_NCNN_SHIM_MODELBIN_H

#include "mat.h"

namespace ncnn {

class ModelBin
{
public:
    virtual ~ModelBin() {}
    virtual Mat load(int w, int type) const = 0;
};

// Hands out the given Mats in order, one per load() call.
class ModelBinFromMatArray : public ModelBin
{
public:
    explicit ModelBinFromMatArray(const Mat* weights) : weights(weights), cursor(0) {}
    virtual Mat load(int w, int type) const
    {
        (void)w;
        (void)type;
        if (!weights) return Mat();
        Mat m = weights[cursor];
        cursor++;
        return m;
    }

private:
    const Mat* weights;
    mutable int cursor;
};

// Reads raw fp32 blobs from a flat float array (the oracle's C entry points
// use this to feed layer weights).
class ModelBinFromFloats : public ModelBin
{
public:
    ModelBinFromFloats(const float* data, size_t count) : data(data), count(count), cursor(0) {}
    virtual Mat load(int w, int type) const
    {
        if ((type != 0 && type != 1) || w <= 0 || cursor + (size_t)w > count) return Mat();
        Mat m(w);
        if (m.empty()) return m;
        for (int i = 0; i < w; i++) ((float*)m.data)[i] = data[cursor + i];
        cursor += (size_t)w;
        return m;
    }

private:
    const float* data;
    size_t count;
    mutable size_t cursor;
};

} // namespace ncnn

#endif
