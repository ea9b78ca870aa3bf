"""GPU: the batched path's tcgen05 GEMM (csrc/batch_kernel.cu, tc_gemm) on its
own, against a plain PyTorch fp32 reference of the same op:
y[t, m] = scale[m] * sum_k W[m, k] x[t, k] with INT8 W tile-packed.

The kernel feeds x as fp16 (11 significant bits) and the exactly dequantised
W to the tensor cores with fp32 accumulation, so the bar is rel_err <= 1e-3
over the output (and cosine >= 0.9999995).  Shapes: every
projection of the model (one tile to four per CTA, slab width 128) and the LM
head (multi-pass, slab width 64), full and ragged batches.
"""
import pytest
import torch

import megaqwen_b200 as mq
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _case(M, K, B, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randint(-128, 128, (M, K), generator=g, device="cuda", dtype=torch.int32).to(torch.int8)
    scale = torch.rand(M, generator=g, device="cuda") * 1e-3 + 1e-4
    x = torch.randn(B, K, generator=g, device="cuda")
    x[:, ::97] *= 30.0   # a few large activations
    y = mq.batch_matmul(mq.pack_tiles(w), scale, x)
    ref = (x.double() @ w.double().t() * scale.double()).float()
    return y, ref


@pytest.mark.parametrize("M,K,B", [(4096, 1024, 64), (1024, 2048, 64), (1024, 3072, 5), (6144, 1024, 33),
                                   (32, 1024, 1), (151936, 1024, 64)])
def test_batch_gemm_matches_fp32(M, K, B):
    y, ref = _case(M, K, B, seed=M + K + B)
    e, c = O.rel_err(ref.cpu(), y.cpu()), O.cosine(ref.cpu(), y.cpu())
    assert e <= 1e-3 and c >= 0.9999995, (e, c)


def test_pack_tiles_layout():
    w = torch.arange(32 * 128, device="cuda", dtype=torch.int32).reshape(32, 128).remainder(251).sub(125).to(torch.int8)
    p = mq.pack_tiles(w).cpu().view(-1)
    wc = w.cpu()
    # block (tile, kb) at ((tile * K/64) + kb) * 1024, inside [8-col group][16 rows][8 bytes]
    for tile in range(2):
        for kb in range(2):
            for kc in range(8):
                for r in range(16):
                    off = ((tile * 2 + kb) * 1024) + kc * 128 + r * 8
                    assert torch.equal(p[off:off + 8], wc[tile * 16 + r, kb * 64 + kc * 8: kb * 64 + kc * 8 + 8])


def test_pack_slabs_layout():
    w = torch.arange(32 * 128, device="cuda", dtype=torch.int32).reshape(32, 128).remainder(251).sub(125).to(torch.int8)
    p = mq.pack_tiles(w, slab_major=True).cpu().view(-1)
    wc = w.cpu()
    # block (kb, tile) at ((kb * rows/16) + tile) * 1024, inside [8-col group][16 rows][8 bytes]
    for tile in range(2):
        for kb in range(2):
            for kc in range(8):
                for r in range(16):
                    off = ((kb * 2 + tile) * 1024) + kc * 128 + r * 8
                    assert torch.equal(p[off:off + 8], wc[tile * 16 + r, kb * 64 + kc * 8: kb * 64 + kc * 8 + 8])


def test_pack_slabs_256_layout():
    w = torch.randint(-128, 128, (48, 512), device="cuda", dtype=torch.int32).to(torch.int8)
    p = mq.pack_tiles(w, slab_major=True, block_k=256).cpu().view(-1)
    wc = w.cpu()
    # block (kb, tile) at ((kb * rows/16) + tile) * 16 * 256, inside [8-col group][16 rows][8 bytes]
    for tile in range(3):
        for kb in range(2):
            for kc in range(32):
                for r in (0, 7, 15):
                    off = ((kb * 3 + tile) * 4096) + kc * 128 + r * 8
                    assert torch.equal(p[off:off + 8], wc[tile * 16 + r, kb * 256 + kc * 8: kb * 256 + kc * 8 + 8])
