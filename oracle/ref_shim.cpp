// TEST INFRASTRUCTURE ONLY -- builds the reference's own CPU expert math into oracle/_ref/ so the
// plain-C oracle can be pinned against it. This file holds no reference code: it includes
// kernels/cpu_avx2/ft_core.h from the reference tree unchanged (its functions live in an anonymous
// namespace, so they are reachable only from a translation unit that includes the header) and
// exports thin extern "C" wrappers around them.
#include "ft_core.h"

#include <cstring>

extern "C" {

void refshim_init() { init_perm(); init_tables(); }

// ft_core.h:65-73
uint16_t refshim_state(const uint16_t* tile, int t) { return state_scalar(tile, t); }

// ft_core.h:75-79
int refshim_bytesum(uint16_t st) { return bytesum(st); }

// ft_core.h:82 (fp16-valued float)
float refshim_weight(uint16_t st) { return w_gpu(st); }

// ft_core.h:48-61
int refshim_perm(int i) { return PERM[i]; }

// ft_core.h:977-992 -> W [k][n] fp32 (fp16-valued)
void refshim_dense_weights(const uint8_t* trellis, int k, int n, float* W)
{
    Mat m{trellis, nullptr, nullptr, k, n};
    std::vector<float> v = dense_weights(m);
    std::memcpy(W, v.data(), v.size() * sizeof(float));
}

// ft_core.h:97-110
void refshim_prep_block(const float* x, const uint16_t* suh, float* xt) { prep_block(x, suh, xt); }
void refshim_out_block(float* y, const uint16_t* svh) { out_block(y, svh); }

// ft_core.h:123-133
float refshim_act(float g, float u, float limit)
{
    const float keep = g_act_limit;
    g_act_limit = limit;
    const float r = act_gu(g, u);
    g_act_limit = keep;
    return r;
}

// ft_core.h:1004-1011 (the reference fixes I = 2048); x [H] fp16-valued -> y [H]
int refshim_ref_expert(const uint8_t* g, const uint8_t* u, const uint8_t* d, const uint16_t* suh_g,
                       const uint16_t* svh_g, const uint16_t* suh_u, const uint16_t* svh_u,
                       const uint16_t* suh_d, const uint16_t* svh_d, int H, int I, const float* x,
                       float limit, float* y)
{
    if (I != 2048) return -1;
    Expert E;
    E.g = {g, suh_g, svh_g, H, I};
    E.u = {u, suh_u, svh_u, H, I};
    E.d = {d, suh_d, svh_d, I, H};
    std::vector<float> W[3] = {dense_weights(E.g), dense_weights(E.u), dense_weights(E.d)};
    const float keep = g_act_limit;
    g_act_limit = limit;
    ref_expert(E, W, x, y);
    g_act_limit = keep;
    return 0;
}

}  // extern "C"
