"""GPU: the full 28-layer Qwen3-0.6B (seeded synthetic weights), 200 greedy
steps with on-device token feedback, against the CPU oracle teacher-forced on
the GPU's own token sequence.  Bar: >= 95 % of the 200 next-token choices
agree, and the logits of a 201st step -- the oracle running on the kernel's own
KV cache, so both sides see identical inputs -- agree to rel_err <= 1e-2,
cosine >= 0.9998."""
import pytest
import torch

import megaqwen_b200 as mq
from oracle import oracle as O
from test_gpu_parity import build_int8, close

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def test_full_model_200_steps():
    L, steps, start = 28, 200, 4242
    st = mq.make_synthetic_state(seed=0, num_layers=L)
    dec = build_int8(st, L, 256)
    toks = dec.decode_steps(start, steps).cpu().tolist()
    dec.check_device()
    orc = O.OracleDecoder(st, L, max_seq_len=256)
    inputs = [start] + toks[:-1]
    agree = 0
    for i, t_in in enumerate(inputs):
        agree += int(orc.decode_step(t_in) == toks[i])
    assert agree >= 0.95 * steps, f"{agree}/{steps}"
    # Final step on identical inputs: the oracle takes the kernel's KV cache (200
    # positions written by the kernel), so the comparison is one step's parity and
    # not the drift of two independently accumulated caches.
    orc.k_cache[:, :, :steps] = dec.k_cache[:, :, :steps].cpu()
    orc.v_cache[:, :, :steps] = dec.v_cache[:, :, :steps].cpu()
    lg = torch.empty(mq.CFG.vocab_size, dtype=torch.float32, device="cuda")
    dec.decode_steps(toks[-1], 1, logits=lg)
    _, l_o, _ = orc.step(toks[-1], want_logits=True)
    close(l_o, lg.cpu())
