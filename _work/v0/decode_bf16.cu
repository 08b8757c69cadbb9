// BF16 decode megakernel for the Qwen3.5-0.8B hybrid network: one persistent cooperative
// launch runs all 24 layers and the LM-head arg-max for one or many tokens.
//
// Replaces models/qwen35_0p8b/kernel.cu (decode_kernel :820-904, lm_head_kernel :747-814,
// launch_decode :910-1020) of the reference.  Work split, per stage:
//   A  RMSNorm -> fused input projection rows, a contiguous row range per CTA
//   B  DeltaNet: every (head, value-row) of the 16 x 128 x 128 f32 state is one warp task
//      spread over all CTAs;  attention: split-KV scores (B1) then P.V partials (B2)
//   C  gated norm / partial merge -> output projection + residual
//   D  RMSNorm -> gate/up rows with fused SiLU*up      E  down projection + residual
// followed by the LM head, whose arg-max takes the lowest index among equal bf16 maxima.
#include "decode_bf16.cuh"

#include <cooperative_groups.h>

namespace q35 {

// 1 / theta^(2i/64), i = 0..31, theta = 1e7 (kernel.cu:483-490 computes it with powf per call);
// filled by the host from a double-precision pow so that it equals torch's f32 table bit for bit.
__constant__ float c_rope_inv_freq[FA_ROT / 2];

#define Q35_SYNC()                          \
    do {                                    \
        if (!grid_sync(bar, &s_flag)) return; \
    } while (0)

__global__ void __launch_bounds__(NTHREADS, 1) decode_bf16_kernel(const DecodeArgs a) {
    __shared__ LayerRec s_layers[NUM_LAYERS];
    __shared__ __align__(16) bf16 s_x[INTER];
    __shared__ float s_red[NWARPS];
    __shared__ float s_part[1024];
    __shared__ __align__(16) float s_qk[2][2][DN_K];
    __shared__ float s_hd[2][2];
    __shared__ __align__(16) float s_q[FA_GQA][FA_HEAD_DIM];
    __shared__ __align__(16) float s_kcur[FA_HEAD_DIM];
    __shared__ float s_p[FA_GQA][256];
    __shared__ float s_ml[FA_GQA][2];
    __shared__ int s_flag;
    __shared__ int s_tok;

    Workspace* ws = a.ws;
    const int b = blockIdx.x, G = gridDim.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (ld_volatile(&ws->err) != 0) return;   // sticky error from an earlier launch
    GridBar bar;
    bar.counter = &ws->bar_counter;
    bar.gen = &ws->bar_gen;
    bar.err = &ws->err;
    bar.nblocks = (unsigned)G;
    bar.cur = *reinterpret_cast<volatile unsigned*>(&ws->bar_gen);

    for (int i = tid; i < NUM_LAYERS * (int)(sizeof(LayerRec) / 16); i += NTHREADS)
        reinterpret_cast<uint4*>(s_layers)[i] = __ldg(reinterpret_cast<const uint4*>(a.layers) + i);
    __syncthreads();

    int tok = a.token_in ? __ldg(a.token_in) : a.token_imm;

    for (int step = 0; step < a.n_steps; ++step) {
        if (a.forced_ids) tok = __ldg(a.forced_ids + step);
        if (tok < 0 || tok >= VOCAB) { if (tid == 0) atomicCAS(&ws->err, 0, (int)ERR_BAD_ARG); tok = 0; }
        const int pos = a.position + step;
        const bool last_step = (step == a.n_steps - 1);
        int i_dn = 0, i_fa = 0;

        const int n_layers = a.dbg_num_layers > 0 ? a.dbg_num_layers : NUM_LAYERS;
        for (int layer = 0; layer < n_layers; ++layer) {
            const LayerRec& L = s_layers[layer];
            const bf16* hin = (layer == 0) ? (a.embed + (size_t)tok * HIDDEN)
                                           : (a.dbg_teacher ? a.dbg_teacher + layer * HIDDEN : ws->h2);
            const bf16* w_post; const bf16* w_gate; const bf16* w_up; const bf16* w_down; const bf16* w_out;

            // ================= stage A: input norm + fused projection =================
            rmsnorm_to_smem(hin, (const bf16*)L.p[0], s_x, s_red);
            __syncthreads();
            if (L.type == 0) {
                const uint4* wqkv = (const uint4*)L.p[DN_QKV]; const uint4* wz = (const uint4*)L.p[DN_Z];
                const uint4* wb = (const uint4*)L.p[DN_B];     const uint4* wa = (const uint4*)L.p[DN_A];
                cta_gemv<HIDDEN, 1, 2, 1>(part_begin(DN_PROJ_ROWS, b, G), part_begin(DN_PROJ_ROWS, b + 1, G), s_x, s_part,
                    [&](int u, int) -> const uint4* {
                        if (u < DN_CONV_CH) return wqkv + (size_t)u * (HIDDEN / 8);
                        if (u < DN_CONV_CH + DN_V_SIZE) return wz + (size_t)(u - DN_CONV_CH) * (HIDDEN / 8);
                        if (u < DN_CONV_CH + DN_V_SIZE + DN_HEADS) return wb + (size_t)(u - DN_CONV_CH - DN_V_SIZE) * (HIDDEN / 8);
                        return wa + (size_t)(u - DN_CONV_CH - DN_V_SIZE - DN_HEADS) * (HIDDEN / 8);
                    },
                    [&](int u, const float* s) { ws->xa[u] = f2bf(s[0]); });
                w_post = (const bf16*)L.p[DN_POST_NORM]; w_gate = (const bf16*)L.p[DN_GATE]; w_up = (const bf16*)L.p[DN_UP];
                w_down = (const bf16*)L.p[DN_DOWN]; w_out = (const bf16*)L.p[DN_OUT];
            } else {
                const uint4* wq = (const uint4*)L.p[FA_Q]; const uint4* wk = (const uint4*)L.p[FA_K]; const uint4* wv = (const uint4*)L.p[FA_V];
                cta_gemv<HIDDEN, 1, 2, 1>(part_begin(FA_PROJ_ROWS, b, G), part_begin(FA_PROJ_ROWS, b + 1, G), s_x, s_part,
                    [&](int u, int) -> const uint4* {
                        if (u < FA_QPROJ) return wq + (size_t)u * (HIDDEN / 8);
                        if (u < FA_QPROJ + FA_KV_SIZE) return wk + (size_t)(u - FA_QPROJ) * (HIDDEN / 8);
                        return wv + (size_t)(u - FA_QPROJ - FA_KV_SIZE) * (HIDDEN / 8);
                    },
                    [&](int u, const float* s) { ws->xa[u] = f2bf(s[0]); });
                w_post = (const bf16*)L.p[FA_POST_NORM]; w_gate = (const bf16*)L.p[FA_GATE]; w_up = (const bf16*)L.p[FA_UP];
                w_down = (const bf16*)L.p[FA_DOWN]; w_out = (const bf16*)L.p[FA_O];
            }
            Q35_SYNC();

            if (L.type == 0) {
                // ================= stage B (DeltaNet): conv, norms, recurrence =================
                const bf16* conv_w = (const bf16*)L.p[DN_CONV];
                float* conv = a.conv_bufs + (size_t)i_dn * DN_CONV_CH * 4;
                float* state = a.dn_states + (size_t)i_dn * DN_HEADS * DN_V * DN_K;
                const int u0 = part_begin(DN_V_SIZE, b, G), u1 = part_begin(DN_V_SIZE, b + 1, G);
                const int hlo = u0 >> 7, hhi = (u1 > u0) ? ((u1 - 1) >> 7) : hlo;   // at most two heads per CTA
                {
                    const int slot = tid >> 8, cl = tid & 255, isk = cl >> 7, i = cl & 127;
                    const bool act = (u1 > u0) && (hlo + slot <= hhi);
                    float c = 0.f, sq = 0.f;
                    if (act) {
                        const int ch = isk * DN_QK_SIZE + (hlo + slot) * DN_K + i;
                        const float4 st = ld_cg(reinterpret_cast<const float4*>(conv) + ch);
                        c = conv_silu(conv_w, ch, st, ld_cg_bf16(ws->xa + ch));
                        sq = rbf(c * c);
                    }
                    const float wsum = warp_sum(sq);
                    if (lane == 0) s_red[warp] = wsum;
                    __syncthreads();
                    if (act) {
                        const int g4 = (tid >> 7) * 4;
                        float tot = ((s_red[g4] + s_red[g4 + 1]) + s_red[g4 + 2]) + s_red[g4 + 3];
                        tot = rbf(tot);
                        tot = rbf(tot + 1e-6f);
                        // torch's CPU rsqrt on a 16-element bf16 tensor takes the scalar path, which rounds
                        // sqrt to bf16 before the reciprocal; decode mirrors that.
                        const float inv = rbf(1.0f / rbf(sqrtf(tot)));
                        float cn = rbf(c * inv);
                        if (!isk) cn = cn * 0.08838834764831845f;     // q * 1/sqrt(128) in f32
                        s_qk[slot][isk][i] = cn;
                    }
                    if (tid < 2 && (u1 > u0) && hlo + tid <= hhi) {
                        const int h = hlo + tid;
                        const float beta = rbf(sigmoid_f(ld_cg_bf16(ws->xa + DN_CONV_CH + DN_V_SIZE + h)));
                        const float x = ld_cg_bf16(ws->xa + DN_CONV_CH + DN_V_SIZE + DN_HEADS + h) + bf2f(((const bf16*)L.p[DN_DTBIAS])[h]);
                        const float sp = (x > 20.f) ? x : log1pf(expf(x));
                        const float g = -expf(bf2f(((const bf16*)L.p[DN_ALOG])[h])) * sp;
                        s_hd[tid][0] = beta;
                        s_hd[tid][1] = expf(g);
                    }
                    __syncthreads();
                }
                for (int u = u0 + warp; u < u1; u += NWARPS) {
                    const int h = u >> 7, v = u & 127, slot = h - hlo;
                    const float4 q4 = *reinterpret_cast<const float4*>(&s_qk[slot][0][lane * 4]);
                    const float4 k4 = *reinterpret_cast<const float4*>(&s_qk[slot][1][lane * 4]);
                    const float beta = s_hd[slot][0], decay = s_hd[slot][1];
                    const int ch = 2 * DN_QK_SIZE + h * DN_V + v;
                    const float vv = conv_silu(conv_w, ch, ld_cg(reinterpret_cast<const float4*>(conv) + ch), ld_cg_bf16(ws->xa + ch));
                    float4* sp = reinterpret_cast<float4*>(state + ((size_t)h * DN_V + v) * DN_K) + lane;
                    float4 s = ld_cg(sp);
                    s.x = __fmul_rn(s.x, decay); s.y = __fmul_rn(s.y, decay); s.z = __fmul_rn(s.z, decay); s.w = __fmul_rn(s.w, decay);
                    float kv = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(s.x, k4.x), __fmul_rn(s.y, k4.y)), __fmul_rn(s.z, k4.z)), __fmul_rn(s.w, k4.w));
                    kv = warp_sum(kv);
                    const float delta = __fmul_rn(__fsub_rn(vv, kv), beta);
                    s.x = __fadd_rn(s.x, __fmul_rn(k4.x, delta)); s.y = __fadd_rn(s.y, __fmul_rn(k4.y, delta));
                    s.z = __fadd_rn(s.z, __fmul_rn(k4.z, delta)); s.w = __fadd_rn(s.w, __fmul_rn(k4.w, delta));
                    float o = __fadd_rn(__fadd_rn(__fadd_rn(__fmul_rn(s.x, q4.x), __fmul_rn(s.y, q4.y)), __fmul_rn(s.z, q4.z)), __fmul_rn(s.w, q4.w));
                    o = warp_sum(o);
                    *sp = s;
                    if (lane == 0) ws->o[u] = f2bf(o);
                }
                Q35_SYNC();

                // ================= stage C (DeltaNet): conv shift, gated norm, out-proj + residual =================
                for (int c = part_begin(DN_CONV_CH, b, G) + tid; c < part_begin(DN_CONV_CH, b + 1, G); c += NTHREADS) {
                    float4 st = ld_cg(reinterpret_cast<const float4*>(conv) + c);
                    st = make_float4(st.y, st.z, st.w, ld_cg_bf16(ws->xa + c));
                    reinterpret_cast<float4*>(conv)[c] = st;
                }
                {
                    const int h = warp;   // 16 warps <-> 16 heads
                    const uint2 orw = ld_cg(reinterpret_cast<const uint2*>(ws->o + h * DN_V) + lane);
                    const uint2 zrw = ld_cg(reinterpret_cast<const uint2*>(ws->xa + DN_CONV_CH + h * DN_V) + lane);
                    const uint2 nrw = __ldg(reinterpret_cast<const uint2*>(L.p[DN_NORM]) + lane);
                    const float ov[4] = {bf_lo(orw.x), bf_hi(orw.x), bf_lo(orw.y), bf_hi(orw.y)};
                    const float zv[4] = {bf_lo(zrw.x), bf_hi(zrw.x), bf_lo(zrw.y), bf_hi(zrw.y)};
                    const float nw[4] = {bf_lo(nrw.x), bf_hi(nrw.x), bf_lo(nrw.y), bf_hi(nrw.y)};
                    const float var = warp_sum(ov[0] * ov[0] + ov[1] * ov[1] + ov[2] * ov[2] + ov[3] * ov[3]) * (1.0f / DN_V);
                    const float r = rsqrt_ieee(var + RMS_EPS);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float n = rbf(ov[i] * r);
                        const float t = rbf(nw[i] * n);
                        s_x[h * DN_V + lane * 4 + i] = f2bf(t * silu_f(zv[i]));
                    }
                }
                ++i_dn;
            } else {
                // ================= stage B1 (attention): q/k norm + RoPE, K/V append, scores =================
                bf16* kc = a.k_cache + (size_t)i_fa * FA_KV_HEADS * a.max_seq_len * FA_HEAD_DIM;
                bf16* vc = a.v_cache + (size_t)i_fa * FA_KV_HEADS * a.max_seq_len * FA_HEAD_DIM;
                const int Lc = pos + 1;
                int nchunk = (Lc + 31) / 32; if (nchunk > ATT_MAX_CHUNKS) nchunk = ATT_MAX_CHUNKS;
                const int clen = (Lc + nchunk - 1) / nchunk;
                const bool att_cta = b < FA_KV_HEADS * nchunk;
                const int kvh = b / nchunk, chunk = b % nchunk;
                const int j0 = chunk * clen, j1 = min(Lc, j0 + clen);
                if (att_cta) {
                    if (warp < FA_GQA + 1) {
                        // warps 0..3: the four query heads of this kv head; warp 4: the new key
                        const bool isq = warp < FA_GQA;
                        const int qh = kvh * FA_GQA + warp;
                        const bf16* src = isq ? (ws->xa + qh * 2 * FA_HEAD_DIM) : (ws->xa + FA_QPROJ + kvh * FA_HEAD_DIM);
                        const bf16* nw = (const bf16*)(isq ? L.p[FA_QNORM] : L.p[FA_KNORM]);
                        float xv[8], ss = 0.f;
#pragma unroll
                        for (int i = 0; i < 8; ++i) { xv[i] = ld_cg_bf16(src + lane + 32 * i); ss += xv[i] * xv[i]; }
                        const float r = rsqrt_ieee(warp_sum(ss) * (1.0f / FA_HEAD_DIM) + RMS_EPS);
#pragma unroll
                        for (int i = 0; i < 8; ++i) xv[i] = rbf((xv[i] * r) * (1.0f + bf2f(nw[lane + 32 * i])));
                        // RoPE on dims [0,64): pairs (d, d+32); here xv[0] is dim `lane`, xv[1] is dim `lane+32`
                        const float ang = (float)pos * c_rope_inv_freq[lane];
                        const float cs = rbf(cosf(ang)), sn = rbf(sinf(ang));
                        const float x1 = xv[0], x2 = xv[1];
                        xv[0] = rbf(rbf(x1 * cs) + rbf(-x2 * sn));
                        xv[1] = rbf(rbf(x2 * cs) + rbf(x1 * sn));
                        float* dst = isq ? s_q[warp] : s_kcur;
#pragma unroll
                        for (int i = 0; i < 8; ++i) dst[lane + 32 * i] = xv[i];
                        if (!isq && pos >= j0 && pos < j1) {
#pragma unroll
                            for (int i = 0; i < 8; ++i) kc[((size_t)kvh * a.max_seq_len + pos) * FA_HEAD_DIM + lane + 32 * i] = f2bf(xv[i]);
                        }
                    } else if (warp == FA_GQA + 1 && pos >= j0 && pos < j1) {
                        const uint4 vr = ld_cg(reinterpret_cast<const uint4*>(ws->xa + FA_QPROJ + FA_KV_SIZE + kvh * FA_HEAD_DIM) + lane);
                        reinterpret_cast<uint4*>(vc + ((size_t)kvh * a.max_seq_len + pos) * FA_HEAD_DIM)[lane] = vr;
                    }
                    __syncthreads();
                    float qr[FA_GQA][8];
#pragma unroll
                    for (int g = 0; g < FA_GQA; ++g)
#pragma unroll
                        for (int i = 0; i < 8; ++i) qr[g][i] = s_q[g][lane * 8 + i];
                    for (int j = j0 + warp; j < j1; j += NWARPS) {
                        float kf[8];
                        if (j == pos) {
#pragma unroll
                            for (int i = 0; i < 8; ++i) kf[i] = s_kcur[lane * 8 + i];
                        } else {
                            const uint4 kr = ld_cg(reinterpret_cast<const uint4*>(kc + ((size_t)kvh * a.max_seq_len + j) * FA_HEAD_DIM) + lane);
                            kf[0] = bf_lo(kr.x); kf[1] = bf_hi(kr.x); kf[2] = bf_lo(kr.y); kf[3] = bf_hi(kr.y);
                            kf[4] = bf_lo(kr.z); kf[5] = bf_hi(kr.z); kf[6] = bf_lo(kr.w); kf[7] = bf_hi(kr.w);
                        }
#pragma unroll
                        for (int g = 0; g < FA_GQA; ++g) {
                            float d = 0.f;
#pragma unroll
                            for (int i = 0; i < 8; ++i) d = fmaf(qr[g][i], kf[i], d);
                            d = warp_sum(d);
                            if (lane == 0) ws->scores[kvh * FA_GQA + g][j] = rbf(d) * 0.0625f;
                        }
                    }
                }
                Q35_SYNC();

                // ================= stage B2 (attention): softmax statistics, P.V partials =================
                if (att_cta) {
                    if (warp < FA_GQA) {
                        const float* sc = ws->scores[kvh * FA_GQA + warp];
                        float mx = -INFINITY;
                        for (int j = lane; j < Lc; j += 32) mx = fmaxf(mx, ld_cg(sc + j));
                        mx = warp_max(mx);
                        float sm = 0.f;
                        for (int j = lane; j < Lc; j += 32) sm += expf(ld_cg(sc + j) - mx);
                        sm = warp_sum(sm);
                        if (lane == 0) { s_ml[warp][0] = mx; s_ml[warp][1] = sm; }
                    }
                    __syncthreads();
                    const int g = tid >> 7, d2 = tid & 127;       // 4 heads x 128 threads, 2 dims each
                    float acc0 = 0.f, acc1 = 0.f;
                    for (int t0 = j0; t0 < j1; t0 += 256) {
                        const int tn = min(256, j1 - t0);
                        __syncthreads();
                        for (int i = tid; i < FA_GQA * tn; i += NTHREADS) {
                            const int gg = i / tn, jj = i % tn;
                            s_p[gg][jj] = rbf(expf(ld_cg(ws->scores[kvh * FA_GQA + gg] + t0 + jj) - s_ml[gg][0]) / s_ml[gg][1]);
                        }
                        __syncthreads();
                        const uint32_t* vb = reinterpret_cast<const uint32_t*>(vc + ((size_t)kvh * a.max_seq_len + t0) * FA_HEAD_DIM) + d2;
#pragma unroll 4
                        for (int jj = 0; jj < tn; ++jj) {
                            const uint32_t vr = ld_cg(vb + (size_t)jj * (FA_HEAD_DIM / 2));
                            const float p = s_p[g][jj];
                            acc0 = fmaf(p, bf_lo(vr), acc0);
                            acc1 = fmaf(p, bf_hi(vr), acc1);
                        }
                    }
                    float2* dst = reinterpret_cast<float2*>(ws->att_part[chunk][kvh * FA_GQA + g]) + d2;
                    *dst = make_float2(acc0, acc1);
                }
                Q35_SYNC();

                // ================= stage C (attention): merge partials, sigmoid gate =================
                {
                    const int qh = tid >> 6, d = (tid & 63) * 4;          // 8 heads x 64 threads x 4 dims
                    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                    for (int c = 0; c < nchunk; ++c) {
                        const float4 pv = ld_cg(reinterpret_cast<const float4*>(&ws->att_part[c][qh][d]));
                        acc.x += pv.x; acc.y += pv.y; acc.z += pv.z; acc.w += pv.w;
                    }
                    const uint2 gr = ld_cg(reinterpret_cast<const uint2*>(ws->xa + qh * 2 * FA_HEAD_DIM + FA_HEAD_DIM + d));
                    const float gv[4] = {bf_lo(gr.x), bf_hi(gr.x), bf_lo(gr.y), bf_hi(gr.y)};
                    const float av[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) s_x[qh * FA_HEAD_DIM + d + i] = f2bf(rbf(av[i]) * rbf(sigmoid_f(gv[i])));
                }
                ++i_fa;
            }
            __syncthreads();
            // ---- stage C tail: output projection (K = 2048) + residual ----
            cta_gemv<2048, 2, 1, 1>(part_begin(HIDDEN, b, G), part_begin(HIDDEN, b + 1, G), s_x, s_part,
                [&](int u, int) -> const uint4* { return reinterpret_cast<const uint4*>(w_out) + (size_t)u * (2048 / 8); },
                [&](int u, const float* s) { ws->h1[u] = f2bf(ld_cg_bf16(hin + u) + rbf(s[0])); });
            Q35_SYNC();

            // ================= stage D: post norm, gate/up with SiLU*up =================
            rmsnorm_to_smem(ws->h1, w_post, s_x, s_red);
            __syncthreads();
            cta_gemv<HIDDEN, 1, 1, 2>(part_begin(INTER, b, G), part_begin(INTER, b + 1, G), s_x, s_part,
                [&](int u, int m) -> const uint4* { return reinterpret_cast<const uint4*>(m ? w_up : w_gate) + (size_t)u * (HIDDEN / 8); },
                [&](int u, const float* s) { ws->m[u] = f2bf(rbf(silu_f(rbf(s[0]))) * rbf(s[1])); });
            Q35_SYNC();

            // ================= stage E: down projection + residual =================
            for (int i = tid; i < INTER / 8; i += NTHREADS)
                reinterpret_cast<uint4*>(s_x)[i] = ld_cg(reinterpret_cast<const uint4*>(ws->m) + i);
            __syncthreads();
            cta_gemv<INTER, 2, 1, 1>(part_begin(HIDDEN, b, G), part_begin(HIDDEN, b + 1, G), s_x, s_part,
                [&](int u, int) -> const uint4* { return reinterpret_cast<const uint4*>(w_down) + (size_t)u * (INTER / 8); },
                [&](int u, const float* s) {
                    const bf16 hv = f2bf(ld_cg_bf16(ws->h1 + u) + rbf(s[0]));
                    ws->h2[u] = hv;
                    if (last_step && a.dbg_hidden) a.dbg_hidden[layer * HIDDEN + u] = hv;
                    if (last_step && layer == NUM_LAYERS - 1 && a.hidden_out) a.hidden_out[u] = hv;
                });
            Q35_SYNC();
        }

        // ================= LM head: final norm, 248320 x 1024 GEMV, arg-max =================
        if (!a.lm_last_only || last_step) {
            rmsnorm_to_smem(ws->h2, a.final_norm, s_x, s_red);
            __syncthreads();
            float best = -INFINITY;
            int best_i = 0x7fffffff;
            float* lg = (last_step ? a.logits_out : nullptr);
            cta_gemv<HIDDEN, 1, 2, 1>(part_begin(VOCAB, b, G), part_begin(VOCAB, b + 1, G), s_x, s_part,
                [&](int u, int) -> const uint4* { return reinterpret_cast<const uint4*>(a.lm_head) + (size_t)u * (HIDDEN / 8); },
                [&](int u, const float* s) {
                    const float v = rbf(s[0]);
                    if (lg) lg[u] = v;
                    if (v > best || (v == best && u < best_i)) { best = v; best_i = u; }
                });
            // lane 0 of every warp holds that warp's best; reduce in the CTA, publish, reduce over CTAs
            if (lane == 0) { s_part[warp] = best; reinterpret_cast<int*>(s_part)[NWARPS + warp] = best_i; }
            __syncthreads();
            if (tid == 0) {
                float bv = s_part[0]; int bi = reinterpret_cast<int*>(s_part)[NWARPS];
                for (int w = 1; w < NWARPS; ++w) {
                    const float v = s_part[w]; const int i = reinterpret_cast<int*>(s_part)[NWARPS + w];
                    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
                }
                ws->lm_val[b] = bv; ws->lm_idx[b] = bi;
            }
            Q35_SYNC();
            if (warp == 0) {
                float bv = -INFINITY; int bi = 0x7fffffff;
                for (int c = lane; c < G; c += 32) {
                    const float v = ld_cg(ws->lm_val + c); const int i = (int)ld_cg(reinterpret_cast<const uint32_t*>(ws->lm_idx) + c);
                    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float v = __shfl_xor_sync(0xffffffffu, bv, o); const int i = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (v > bv || (v == bv && i < bi)) { bv = v; bi = i; }
                }
                if (lane == 0) s_tok = bi;
            }
            __syncthreads();
            tok = s_tok;
            if (b == 0 && tid == 0) {
                if (a.out_tokens) a.out_tokens[step] = tok;
                if (last_step && a.out_token) *a.out_token = tok;
            }
        }
    }
}

}  // namespace q35

// ======================================= host side ==========================================
#include <cmath>
#include <cstdlib>
#include <mutex>

#include "runtime.h"

namespace q35 {

static void rope_table(float* t) {
    for (int i = 0; i < FA_ROT / 2; ++i) {
        const float e = (float)(2 * i) / (float)FA_ROT;
        const float p = (float)std::pow(1.0e7, (double)e);
        t[i] = 1.0f / p;
    }
}

static int decode_grid() {
    // one persistent CTA per SM; MEGAKERNEL_DECODE_BLOCKS overrides (same knob as the reference, kernel.cu:926-943)
    int g = device_sm_count();
    if (const char* s = getenv("MEGAKERNEL_DECODE_BLOCKS")) {
        const int v = atoi(s);
        if (v >= 32 && v <= g) g = v;
    }
    return g;
}

static int launch_decode_impl(const DecodeArgs& in, cudaStream_t stream) {
    static std::once_flag once[64];
    static bool ready[64] = {};
    int dev = 0;
    Q35_CUDA_OK(cudaGetDevice(&dev));
    std::call_once(once[dev & 63], [&] {
        float t[FA_ROT / 2];
        rope_table(t);
        int nb = 0;
        if (cudaMemcpyToSymbol(c_rope_inv_freq, t, sizeof(t)) == cudaSuccess &&
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, decode_bf16_kernel, NTHREADS, 0) == cudaSuccess && nb >= 1)
            ready[dev & 63] = true;
    });
    if (!ready[dev & 63]) { set_error("decode kernel cannot be made resident on this device"); return QWEN35_ERR_CUDA; }

    DecodeArgs a = in;
    if (a.n_steps <= 0) return QWEN35_OK;
    if (!a.layers || !a.embed || !a.final_norm || !a.lm_head || !a.k_cache || !a.v_cache || !a.dn_states || !a.conv_bufs) {
        set_error("null tensor pointer");
        return QWEN35_ERR_BAD_ARG;
    }
    if (a.position < 0 || a.max_seq_len <= 0 || a.position + a.n_steps > a.max_seq_len || a.max_seq_len > MAX_CTX) {
        set_error("position %d + %d steps exceeds max_seq_len %d (library limit %d)", a.position, a.n_steps, a.max_seq_len, MAX_CTX);
        return QWEN35_ERR_BAD_ARG;
    }
    if (!a.token_in && !a.forced_ids && (a.token_imm < 0 || a.token_imm >= VOCAB)) {
        set_error("token id %d out of range", a.token_imm);
        return QWEN35_ERR_BAD_ARG;
    }
    a.ws = get_workspace();
    if (!a.ws) return QWEN35_ERR_CUDA;
    void* params[] = {(void*)&a};
    Q35_CUDA_OK(cudaLaunchCooperativeKernel((const void*)decode_bf16_kernel, dim3(decode_grid()), dim3(NTHREADS), params, 0, stream));
    g_launches.fetch_add(1);
    return QWEN35_OK;
}

}  // namespace q35

extern "C" int launch_decode(
    int input_token_id, int* output_token_id,
    const void* embed_weight, const LayerWeights* layer_weights,
    const void* final_norm_weight, const void* lm_head_weight,
    void* fa_k_cache, void* fa_v_cache, void* dn_states, void* conv_bufs,
    void* hidden_buffer, void*, void*, void*, void*, void*, void*, void*, void*, void*, void*,
    unsigned int*, unsigned int*, float*, int*, unsigned int*,
    int position, int max_seq_len, qwen35_stream_t stream) {
    q35::DecodeArgs a = {};
    a.layers = reinterpret_cast<const q35::LayerRec*>(layer_weights);
    a.embed = (const q35::bf16*)embed_weight;
    a.final_norm = (const q35::bf16*)final_norm_weight;
    a.lm_head = (const q35::bf16*)lm_head_weight;
    a.k_cache = (q35::bf16*)fa_k_cache;
    a.v_cache = (q35::bf16*)fa_v_cache;
    a.dn_states = (float*)dn_states;
    a.conv_bufs = (float*)conv_bufs;
    a.token_imm = input_token_id;
    a.out_token = output_token_id;
    a.hidden_out = (q35::bf16*)hidden_buffer;
    a.position = position;
    a.max_seq_len = max_seq_len;
    a.n_steps = 1;
    return q35::launch_decode_impl(a, (cudaStream_t)stream);
}

extern "C" int qwen35_b200_decode_steps(const Qwen35DecodeArgs* in, qwen35_stream_t stream) {
    if (!in) { q35::set_error("null args"); return QWEN35_ERR_BAD_ARG; }
    q35::DecodeArgs a = {};
    a.layers = reinterpret_cast<const q35::LayerRec*>(in->layer_weights);
    a.embed = (const q35::bf16*)in->embed_weight;
    a.final_norm = (const q35::bf16*)in->final_norm_weight;
    a.lm_head = (const q35::bf16*)in->lm_head_weight;
    a.k_cache = (q35::bf16*)in->fa_k_cache;
    a.v_cache = (q35::bf16*)in->fa_v_cache;
    a.dn_states = (float*)in->dn_states;
    a.conv_bufs = (float*)in->conv_bufs;
    a.token_in = in->token_in;
    a.token_imm = in->token_imm;
    a.forced_ids = in->forced_ids;
    a.out_token = in->out_token;
    a.out_tokens = in->out_tokens;
    a.logits_out = in->logits_out;
    a.hidden_out = (q35::bf16*)in->hidden_out;
    a.dbg_hidden = (q35::bf16*)in->dbg_hidden;
    a.dbg_teacher = (const q35::bf16*)in->dbg_teacher;
    a.position = in->position;
    a.max_seq_len = in->max_seq_len;
    a.n_steps = in->n_steps;
    a.lm_last_only = in->lm_last_only;
    a.dbg_num_layers = in->dbg_num_layers;
    return q35::launch_decode_impl(a, (cudaStream_t)stream);
}

extern "C" int qwen35_b200_rope_inv_freq(float* host_out32) {
    if (!host_out32) return QWEN35_ERR_BAD_ARG;
    q35::rope_table(host_out32);
    return QWEN35_OK;
}

// Debug: copy one workspace vector to the host after synchronising the device.
// which: 0 = xa (8224 bf16), 1 = o (2048 bf16), 2 = h1 (1024 bf16), 3 = m (3584 bf16), 4 = h2 (1024 bf16)
extern "C" int qwen35_b200_debug_read(int which, void* host_out) {
    using namespace q35;
    Workspace* ws = get_workspace();
    if (!ws || !host_out) return QWEN35_ERR_BAD_ARG;
    const void* src; size_t n;
    switch (which) {
        case 0: src = ws->xa; n = DN_PROJ_ROWS * 2; break;
        case 1: src = ws->o; n = DN_V_SIZE * 2; break;
        case 2: src = ws->h1; n = HIDDEN * 2; break;
        case 3: src = ws->m; n = INTER * 2; break;
        case 4: src = ws->h2; n = HIDDEN * 2; break;
        default: return QWEN35_ERR_BAD_ARG;
    }
    Q35_CUDA_OK(cudaDeviceSynchronize());
    Q35_CUDA_OK(cudaMemcpy(host_out, src, n, cudaMemcpyDeviceToHost));
    return QWEN35_OK;
}
