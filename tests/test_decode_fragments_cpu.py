"""A CPU model of the fused decode step's tensor-core data path, checked
against a direct computation.

The consumer warps of decode_step_kernel (ryzenai-npu-lab_b200/csrc/b2_attn.cu,
step_consumer) read 64 x 64 bf16 K/V tiles that TMA wrote with the 128-byte
swizzle, fetch fragments with ldmatrix (.trans for V) and multiply with
mma.sync m16n8k16; the probabilities reach the second product through warp
shuffles and byte permutes.  This model replays exactly that index
arithmetic lane by lane with numpy, following the PTX ISA's fragment layouts:

  swizzle     byte offset of (row r, 16-byte chunk c) = 128 r + 16 (c ^ (r % 8))
  ldmatrix    lanes 8i..8i+7 give the row addresses of 8x8 matrix i; lane T
              receives elements (T / 4, 2 (T % 4) .. +1) of each matrix, or with
              .trans elements (2 (T % 4) .. +1, T / 4)
  mma A       a0 (g, 2t..2t+1)  a1 (g+8, 2t..)  a2 (g, 2t+8..)  a3 (g+8, 2t+8..)
  mma B       b0 (k 2t..2t+1, n g)  b1 (k 2t+8..2t+9, n g)
  mma C       c0 c1 (g, 2t 2t+1)  c2 c3 (g+8, 2t 2t+1)        g = lane / 4, t = lane % 4

With `tokens` = 1 the model is the shipped kernel: the N = 8 side carries the
two query heads of a GQA pair and six zero columns.  With tokens = 2..4 it is
the multi-token layout (column n = 2 * token + head, lane t owning token t's
state, causal masks per token, the P^T shuffle reading lanes 8t + token and
8t + 4 + token), checked here before a kernel uses it.
"""
import numpy as np
import pytest
import torch

LANES = 32


def bf16(x):
    """Round-to-nearest-even to bf16, returned as float32."""
    return torch.from_numpy(np.asarray(x, dtype=np.float32)).to(torch.bfloat16).float().numpy()


def swizzled(tile):
    """The TMA image of a [64, 64] bf16 tile with the 128-byte swizzle: a flat
    array of 4096 elements indexed by byte offset / 2."""
    flat = np.zeros(64 * 64, dtype=np.float32)
    for r in range(64):
        for c in range(8):
            off = r * 128 + ((c ^ (r & 7)) << 4)
            flat[off // 2: off // 2 + 8] = tile[r, 8 * c: 8 * c + 8]
    return flat


def ldmatrix_x4(flat, addrs, trans=False):
    """addrs[lane] = byte address of the 8-element row that lane supplies.
    Returns regs[4][32][2]: each lane's two bf16 halves (low, high) per matrix."""
    regs = np.zeros((4, LANES, 2), dtype=np.float32)
    for i in range(4):
        rows = [flat[addrs[8 * i + r] // 2: addrs[8 * i + r] // 2 + 8] for r in range(8)]
        for lane in range(LANES):
            if trans:
                regs[i, lane] = [rows[2 * (lane % 4)][lane // 4], rows[2 * (lane % 4) + 1][lane // 4]]
            else:
                regs[i, lane] = rows[lane // 4][2 * (lane % 4): 2 * (lane % 4) + 2]
    return regs


def mma_m16n8k16(c, a, b):
    """c[32][4] += A . B with A from a[4][32][2] and B from b[2][32][2] (fp32 accumulate)."""
    A = np.zeros((16, 16), dtype=np.float32)
    B = np.zeros((16, 8), dtype=np.float32)
    for lane in range(LANES):
        g, t = lane // 4, lane % 4
        A[g, 2 * t: 2 * t + 2] = a[0, lane]
        A[g + 8, 2 * t: 2 * t + 2] = a[1, lane]
        A[g, 2 * t + 8: 2 * t + 10] = a[2, lane]
        A[g + 8, 2 * t + 8: 2 * t + 10] = a[3, lane]
        B[2 * t: 2 * t + 2, g] = b[0, lane]
        B[2 * t + 8: 2 * t + 10, g] = b[1, lane]
    C = A.astype(np.float64) @ B.astype(np.float64)
    out = c.copy()
    for lane in range(LANES):
        g, t = lane // 4, lane % 4
        out[lane] += [C[g, 2 * t], C[g, 2 * t + 1], C[g + 8, 2 * t], C[g + 8, 2 * t + 1]]
    return out.astype(np.float32)


def shfl(vals, src):
    """__shfl_sync: lane l receives vals[src[l]] (vals[lane] is a bf16 pair)."""
    return np.stack([vals[s] for s in src])


def consumer_item(k_tiles, v_tiles, q, rows_per_tile, scale_log2, tokens):
    """One item as the four consumer warps run it: q [tokens, 2, 64] (the GQA
    pair of each token), k/v tiles [n][64, 64], rows_per_tile[n] = keys left
    from the tile's first row on (the last token's limit; not clamped to 64).
    Returns per warp the state (m [32][2], l [32][2], o [32][4][4]) in the
    kernel's lane layout; the P^T words are built as __byte_perm(v_lo, v_hi,
    0x5410 or 0x7632) does, taking half (column % 2) of each shuffled word."""
    states = []
    for warp in range(4):
        lanes = np.arange(LANES)
        g, t, j = lanes // 4, lanes % 4, lanes // 8
        # B fragment of Q^T: column n = g is (token g / 2, head g % 2); zero beyond 2 * tokens
        bq = np.zeros((4, 2, LANES, 2), dtype=np.float32)
        for ks in range(4):
            for lane in range(LANES):
                gg, tt = lane // 4, lane % 4
                if gg < 2 * tokens:
                    tok, head = gg // 2, gg % 2
                    bq[ks, 0, lane] = q[tok, head, 16 * ks + 2 * tt: 16 * ks + 2 * tt + 2]
                    bq[ks, 1, lane] = q[tok, head, 16 * ks + 2 * tt + 8: 16 * ks + 2 * tt + 10]
        m = np.full((LANES, 2), -1.0e30, dtype=np.float32)
        l = np.zeros((LANES, 2), dtype=np.float32)
        o = np.zeros((LANES, 4, 4), dtype=np.float32)
        qk_row = 16 * warp + (lanes & 7) + 8 * (j & 1)
        pv_row = 16 * warp + (lanes & 7) + 8 * (j >> 1)
        for kt, vt, rows in zip(k_tiles, v_tiles, rows_per_tile):
            kflat, vflat = swizzled(kt), swizzled(vt)
            c = np.zeros((LANES, 4), dtype=np.float32)
            for ks in range(4):
                chunk = 2 * ks + (j >> 1)
                a = ldmatrix_x4(kflat, qk_row * 128 + ((chunk ^ (qk_row & 7)) << 4))
                c = mma_m16n8k16(c, a, bq[ks])
            valid = rows - 16 * warp
            # lane (g, t): scores of rows g, g+8 for token t, heads 0 and 1;
            # token t sees keys up to its own position: tokens - 1 - t fewer rows
            lane_ok = t < tokens
            vt_tok = valid - (tokens - 1 - t)
            s = np.full((LANES, 2, 2), -np.inf, dtype=np.float32)   # [lane][row g | g+8][head]
            for lane in range(LANES):
                if not lane_ok[lane]:
                    continue
                if g[lane] < vt_tok[lane]:
                    s[lane, 0] = c[lane, 0:2] * scale_log2
                if g[lane] + 8 < vt_tok[lane]:
                    s[lane, 1] = c[lane, 2:4] * scale_log2
            bm = s.max(axis=1)                                        # [lane][head]
            for off in (4, 8, 16):                                    # rows only (same t)
                bm = np.maximum(bm, bm[lanes ^ off])
            mn = np.maximum(m, bm)
            alpha = np.exp2(m - mn)
            m = mn
            p = np.exp2(s - mn[:, None, :])                           # [lane][row][head]
            l = l * alpha + p.sum(axis=1)
            o *= np.stack([alpha[:, 0], alpha[:, 1], alpha[:, 0], alpha[:, 1]], axis=1)[:, None, :]
            pk0, pk1 = bf16(p[:, 0]), bf16(p[:, 1])                   # (head 0, head 1) of rows g, g+8
            tok = g // 2
            v0, v1 = shfl(pk0, 8 * t + tok), shfl(pk0, 8 * t + 4 + tok)
            v2, v3 = shfl(pk1, 8 * t + tok), shfl(pk1, 8 * t + 4 + tok)
            bp = np.zeros((2, LANES, 2), dtype=np.float32)
            for lane in range(LANES):
                if g[lane] < 2 * tokens:
                    half = g[lane] % 2
                    bp[0, lane] = [v0[lane, half], v1[lane, half]]
                    bp[1, lane] = [v2[lane, half], v3[lane, half]]
            for mt in range(4):
                chunk = 2 * mt + (j & 1)
                a = ldmatrix_x4(vflat, pv_row * 128 + ((chunk ^ (pv_row & 7)) << 4), trans=True)
                if valid < 16:     # rows past the end are zeroed (they may hold NaN)
                    for lane in range(LANES):
                        tt = lane % 4
                        for reg, base in ((0, 2 * tt), (1, 2 * tt), (2, 2 * tt + 8), (3, 2 * tt + 8)):
                            a[reg, lane] = [a[reg, lane][e] if base + e < valid else 0.0 for e in range(2)]
                o[:, mt] = mma_m16n8k16(o[:, mt], a, bp)
        states.append((m, l, o))
    return states


def epilogue(states, tokens):
    """The step epilogue's merge of the 4 warps: context [tokens, 2, 64]."""
    ctx = np.zeros((tokens, 2, 64), dtype=np.float32)
    for tok in range(tokens):
        for h in range(2):
            parts = []
            for m, l, o in states:
                lanes = [4 * g + tok for g in range(8)]
                mm = m[lanes[0], h]
                ll = sum(l[x, h] for x in lanes)
                vec = np.zeros(64, dtype=np.float32)
                for g in range(8):
                    lane = 4 * g + tok
                    for mt in range(4):
                        vec[16 * mt + g] = o[lane, mt, h]
                        vec[16 * mt + g + 8] = o[lane, mt, 2 + h]
                parts.append((mm, ll, vec))
            big = max(p[0] for p in parts)
            L = sum(ll * np.exp2(mm - big) for mm, ll, _ in parts)
            O = sum(vec * np.exp2(mm - big) for mm, _, vec in parts)
            ctx[tok, h] = O / L
    return ctx


def reference(q, keys, values, past, tokens, scale):
    """Direct attention: token tok attends keys [0, past + tok] (fp64)."""
    out = np.zeros((tokens, 2, 64))
    for tok in range(tokens):
        n = past + tok + 1
        for h in range(2):
            s = keys[:n].astype(np.float64) @ q[tok, h].astype(np.float64) * scale
            p = np.exp(s - s.max())
            out[tok, h] = (p / p.sum()) @ values[:n].astype(np.float64)
    return out


@pytest.mark.parametrize("tokens", [1, 2, 3, 4])
@pytest.mark.parametrize("past", [0, 5, 60, 63, 64, 100, 125])
def test_fragment_layout_matches_direct_attention(tokens, past):
    rng = np.random.default_rng(1000 * tokens + past)
    total = past + tokens
    ntiles = -(-total // 64)
    keys = bf16(rng.standard_normal((ntiles * 64, 64)))
    values = bf16(rng.standard_normal((ntiles * 64, 64)))
    keys[total:] = np.nan            # stale rows past the end must not reach the output
    values[total:] = np.nan
    q = bf16(rng.standard_normal((tokens, 2, 64)))
    scale = 0.125
    # rows left from each tile on, unclamped, as the producer's StageMeta.rows: the per-token
    # causal offset only bites in the tile where fewer than 16 + tokens rows are left
    rows = [total - 64 * i for i in range(ntiles)]
    states = consumer_item([keys[64 * i: 64 * i + 64] for i in range(ntiles)],
                           [values[64 * i: 64 * i + 64] for i in range(ntiles)],
                           q, rows, scale * np.log2(np.e), tokens)
    got = epilogue(states, tokens)
    want = reference(q, keys, values, past, tokens, scale)
    assert np.isfinite(got).all()
    # P is rounded to bf16 before the second product (as in the kernel): ~2^-8 relative
    np.testing.assert_allclose(got, want, atol=2e-2, rtol=1e-2)


def test_swizzle_is_a_permutation_of_16_byte_chunks():
    offs = sorted(r * 128 + ((c ^ (r & 7)) << 4) for r in range(64) for c in range(8))
    assert offs == list(range(0, 8192, 16))
