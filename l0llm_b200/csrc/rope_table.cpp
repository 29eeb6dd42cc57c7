// Inverse-frequency tables for rotary embeddings: default, linear, YaRN and Llama 3.1 scaling.
// Follows L/RopeFrequencies.cs:67-183 (which mirrors transformers' ROPE_INIT_FUNCTIONS): every value
// is computed in double and rounded to float once.
#include <algorithm>
#include <cmath>

#include "model.h"

namespace l0b {

namespace {

double mscale_of(double scale, double mscale) { return scale <= 1.0 ? 1.0 : 0.1 * mscale * std::log(scale) + 1.0; }

double correction_dim(double rotations, int dim, double theta, double max_position) {
    return dim * std::log(max_position / (rotations * 2 * M_PI)) / (2 * std::log(theta));
}

}  // namespace

l0b_status rope_frequencies(const l0b_model_config& c, std::vector<float>* out, float* attention_factor) {
    const int rot = static_cast<int>(c.head_dim * (c.partial_rotary_factor > 0 ? c.partial_rotary_factor : 1.0));
    L0B_REQUIRE(rot > 0 && rot % 2 == 0, L0B_ERR_OUT_OF_RANGE, "head_dim must be positive and even (rotary dim %d)",
                rot);
    const int half = rot / 2;
    const double theta = c.rope_theta;
    std::vector<double> base(half);
    for (int i = 0; i < half; ++i) base[i] = 1.0 / std::pow(theta, 2.0 * i / rot);
    std::vector<double> res(base);
    double attention = 1.0;
    switch (c.rope_type) {
        case L0B_ROPE_DEFAULT: break;
        case L0B_ROPE_LINEAR:
            for (int i = 0; i < half; ++i) res[i] = base[i] / c.rope_factor;
            break;
        case L0B_ROPE_YARN: {
            const double factor = c.rope_factor;
            const double original = c.rope_original_max_position > 0 ? c.rope_original_max_position
                                                                     : c.max_position_embeddings;
            if (c.rope_attention_factor > 0) attention = c.rope_attention_factor;
            else if (c.rope_mscale > 0 && c.rope_mscale_all_dim > 0)
                attention = mscale_of(factor, c.rope_mscale) / mscale_of(factor, c.rope_mscale_all_dim);
            else attention = mscale_of(factor, 1.0);
            double low = correction_dim(c.rope_beta_fast, rot, theta, original);
            double high = correction_dim(c.rope_beta_slow, rot, theta, original);
            if (c.rope_truncate) {
                low = std::floor(low);
                high = std::ceil(high);
            }
            low = std::max(low, 0.0);
            high = std::min(high, static_cast<double>(rot - 1));
            if (low == high) high += 0.001;
            for (int i = 0; i < half; ++i) {
                const double ramp = std::clamp((i - low) / (high - low), 0.0, 1.0);
                const double extra = 1.0 - ramp;
                const double interp = base[i] / factor;
                res[i] = interp * (1.0 - extra) + base[i] * extra;
            }
            break;
        }
        case L0B_ROPE_LLAMA3: {
            const double original = c.rope_original_max_position > 0 ? c.rope_original_max_position
                                                                     : c.max_position_embeddings;
            const double low_wl = original / c.rope_low_freq_factor;
            const double high_wl = original / c.rope_high_freq_factor;
            for (int i = 0; i < half; ++i) {
                const double f = base[i];
                const double wl = 2 * M_PI / f;
                if (wl < high_wl) res[i] = f;
                else if (wl > low_wl) res[i] = f / c.rope_factor;
                else {
                    const double smooth =
                        (original / wl - c.rope_low_freq_factor) / (c.rope_high_freq_factor - c.rope_low_freq_factor);
                    res[i] = (1 - smooth) * f / c.rope_factor + smooth * f;
                }
            }
            break;
        }
        default: return fail(L0B_ERR_UNSUPPORTED, "rope_scaling type %d is not supported", c.rope_type);
    }
    out->resize(half);
    for (int i = 0; i < half; ++i) (*out)[i] = static_cast<float>(res[i]);
    *attention_factor = static_cast<float>(attention);
    return L0B_OK;
}

}  // namespace l0b

extern "C" L0B_API l0b_status l0b_rope_frequencies(const l0b_model_config* cfg, float* inv_freq, int32_t capacity,
                                                   int32_t* count, float* attention_factor) {
    L0B_REQUIRE(cfg && count && attention_factor, l0b_status::L0B_ERR_ARGUMENT, "null argument");
    std::vector<float> t;
    float att = 1.f;
    L0B_TRY(l0b::rope_frequencies(*cfg, &t, &att));
    *count = static_cast<int32_t>(t.size());
    *attention_factor = att;
    if (inv_freq) {
        L0B_REQUIRE(capacity >= static_cast<int32_t>(t.size()), L0B_ERR_ARGUMENT, "inv_freq holds %d, need %zu",
                    capacity, t.size());
        for (size_t i = 0; i < t.size(); ++i) inv_freq[i] = t[i];
    }
    return L0B_OK;
}
