// ref_gdn.cu -- builds the reference's own CPU GDN functions from its source
// file where it lies (the path is given by the Makefile as REF_GDN_SRC), and
// exports them with a C ABI for the parity tests.  TEST INFRASTRUCTURE ONLY.
//
// Exported:
//   ref_gdn_cpu          -> gdn_cpu          src/gdn_sm75.cu:1078-1106
//   ref_gdn_chunked_cpu  -> gdn_chunked_cpu  src/gdn_sm75.cu:1109-1244
// Both run at the reference's compiled-in shape (Sv=128, Hq=16, Hv=48,
// CS=16, no batch), fp32.  The reference's main() is renamed so it is not
// the library's entry point.
#define main reference_gdn_main
#include REF_GDN_SRC
#undef main

extern "C" int ref_gdn_shape(int* sv, int* hq, int* hv, int* cs) {
    *sv = kSv; *hq = kHq; *hv = kHv; *cs = kCs;
    return 0;
}

static void ref_call(bool chunked, const float* q, const float* k, const float* v,
                     const float* g, const float* b, float* state, float* out, int T,
                     float scale) {
    std::vector<float> vq(q, q + (size_t)T * kHq * kSv);
    std::vector<float> vk(k, k + (size_t)T * kHq * kSv);
    std::vector<float> vv(v, v + (size_t)T * kHv * kSv);
    std::vector<float> vg(g, g + (size_t)T * kHv);
    std::vector<float> vb(b, b + (size_t)T * kHv);
    std::vector<float> vs(state, state + (size_t)kHv * kSv * kSv);
    std::vector<float> vo((size_t)T * kHv * kSv);
    if (chunked) gdn_chunked_cpu(vq, vk, vv, vg, vb, vs, vo, T, scale);
    else gdn_cpu(vq, vk, vv, vg, vb, vs, vo, T, scale);
    std::copy(vs.begin(), vs.end(), state);
    std::copy(vo.begin(), vo.end(), out);
}

extern "C" int ref_gdn_cpu(const float* q, const float* k, const float* v, const float* g,
                           const float* b, float* state, float* out, int T, float scale) {
    if (T < 1) return -1;
    ref_call(false, q, k, v, g, b, state, out, T, scale);
    return 0;
}

extern "C" int ref_gdn_chunked_cpu(const float* q, const float* k, const float* v,
                                   const float* g, const float* b, float* state, float* out,
                                   int T, float scale) {
    if (T < 1) return -1;
    ref_call(true, q, k, v, g, b, state, out, T, scale);
    return 0;
}
