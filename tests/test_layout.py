"""The T2B weight layout on the CPU: a test-side packing written from the
layout's description (``include/t2b.h``: 8 KB blocks of 128 rows x 128 k,
piece p of row r at p*2048 + r*16, even k first inside each 32-bit word,
meta = fp16 scale | (stored zero + 1) << 16) is inverted exactly by
``weights.dequantize``, for a plain matrix and for the fused row orders
(``[q; k; v]`` concatenation and gate/up interleaved in 64-row blocks)."""

import torch

import oracle
from torch2iron_b200 import synth
from torch2iron_b200 import weights as W


def _pack_t2b(lins, block_rows=None, block_stride=0):
    """AutoGPTQ linears -> (qw uint8 [N, K/2], meta int32 [N, K/128]) in the T2B layout,
    rows of part i mapped like the repack kernel: row0 + (n // block_rows) * block_stride + n % block_rows."""
    k = lins[0].in_features
    n_total = sum(l.out_features for l in lins) if block_stride == 0 else 2 * lins[0].out_features
    g = k // 128
    qw = torch.zeros(n_total // 128, g, 4, 128, 16, dtype=torch.uint8)
    meta = torch.zeros(n_total // 128, g, 128, dtype=torch.int64)
    row0 = 0
    for part, lin in enumerate(lins):
        n = lin.out_features
        q = oracle.unpack_autogptq_qweight(lin.qweight, k, n).to(torch.int64)         # [n, k]
        z = oracle.unpack_autogptq_qzeros(lin.qzeros, n).to(torch.int64)              # [G, n] (+1 applied)
        s = lin.scales.contiguous().view(torch.int16).to(torch.int64) & 0xFFFF        # [G, n] fp16 bits
        br = block_rows or n
        base = row0 if block_stride == 0 else part * block_rows
        for r in range(n):
            dst = base + (r // br) * (block_stride or br) + r % br
            nt, rr = dst // 128, dst % 128
            for gg in range(g):
                meta[nt, gg, rr] = s[gg, r] | (z[gg, r] << 16)
                for p in range(4):
                    words = []
                    for j in range(4):
                        ks = gg * 128 + p * 32 + j * 8
                        vals = q[r, ks:ks + 8]
                        w = 0
                        for t in range(4):
                            w |= int(vals[2 * t]) << (4 * t)          # slot t: k 2t
                            w |= int(vals[2 * t + 1]) << (4 * (t + 4))  # slot t+4: k 2t+1
                        words.append(w)
                    qw[nt, gg, p, rr] = torch.tensor(
                        [(wd >> (8 * b)) & 0xFF for wd in words for b in range(4)], dtype=torch.uint8)
        row0 += n
    qw = qw.reshape(-1).view(n_total, k // 2)
    meta = meta.to(torch.int32).reshape(-1).view(n_total, g)
    return W.W4Weight(qw, meta, n_total, k)


def _dense(lin):
    return oracle.autogptq_linear_to_dense(lin.qweight, lin.qzeros, lin.scales)


def test_documented_layout_round_trips_through_dequantize():
    g = torch.Generator().manual_seed(5)
    lin = synth.random_linear(128, 256, g)
    assert torch.equal(W.dequantize(_pack_t2b([lin])), _dense(lin))


def test_fused_row_orders():
    g = torch.Generator().manual_seed(6)
    q, k, v = (synth.random_linear(n, 256, g) for n in (256, 128, 128))
    fused = W.dequantize(_pack_t2b([q, k, v]))
    assert torch.equal(fused, torch.cat([_dense(q), _dense(k), _dense(v)]))
    gate, up = synth.random_linear(128, 256, g), synth.random_linear(128, 256, g)
    paired = W.dequantize(_pack_t2b([gate, up], block_rows=64, block_stride=128))
    want = torch.cat([_dense(gate)[0:64], _dense(up)[0:64], _dense(gate)[64:128], _dense(up)[64:128]])
    assert torch.equal(paired, want)
