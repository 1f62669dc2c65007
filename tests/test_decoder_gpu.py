"""Decoder tail kernels against the reference's PyTorch formulas (decoder.py:65-89).

* ``local_topk``: the masked top-k selection is exact (scores drawn without repeats, so
  torch.topk's choice is unique) and the masked mean equal up to FP32 summation order;
  with repeated scores, frames of equal score carry equal features, so any tie order
  gives the same mean. ``local.float()`` is bit-exact.
* ``decoder_heads``: five BF16 projections with FP32 accumulation against the same
  layers run by cuBLAS under BF16 autocast: only the summation order differs, so a
  hidden value may round to the neighbouring BF16 value; logits are held to 2 BF16 ulps
  of the largest logit, and most of them match exactly.
* The whole decoder (the fused tail) against the unfused PyTorch tail of the same module.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)

from trifusion_b200.decoder import Decoder  # noqa: E402
from trifusion_b200.kernels.native import decoder_heads, local_topk  # noqa: E402
from trifusion_b200.masking import Grids, time_mask  # noqa: E402


def reference_top(local, features, fine_lengths):
    """decoder.py:65-76 verbatim in PyTorch (local BF16 [B,T,2], features BF16 [B,T,256])."""
    tf_ = local.shape[1]
    fine_mask = time_mask(fine_lengths, tf_)
    k = min(25, tf_)
    scores = local.float().masked_fill(~fine_mask.unsqueeze(-1), -torch.inf)
    idx = scores.transpose(1, 2).topk(k, -1).indices
    picked = features.unsqueeze(1).expand(-1, 2, -1, -1).gather(2, idx.unsqueeze(-1).expand(-1, -1, -1, 256))
    valid_k = torch.arange(k, device=local.device)[None, :] < fine_lengths.clamp(max=k)[:, None]
    return (picked.float() * valid_k[:, None, :, None]).sum(2) / valid_k.sum(1)[:, None, None]


def distinct_scores(b, t, gen):
    """BF16 scores of [b, t, 2] with no repeats within a (clip, class) column."""
    pool = torch.arange(0x3000, 0x3000 + 4096, dtype=torch.int32)  # positive BF16 bit patterns
    cols = []
    for _ in range(2 * b):
        bits = pool[torch.randperm(4096, generator=gen)[:t]]
        sign = torch.where(torch.rand(t, generator=gen) < 0.5, 0x8000, 0)
        cols.append(((bits | sign).to(torch.int16)).view(torch.bfloat16))
    return torch.stack(cols, 1).view(t, b, 2).permute(1, 0, 2).contiguous()


@pytest.mark.parametrize("t", [1, 24, 25, 26, 200, 3600])
def test_local_topk_distinct_scores(t):
    gen = torch.Generator().manual_seed(t)
    b = 5
    local = distinct_scores(b, t, gen).cuda()
    features = torch.randn(b, t, 256, generator=gen).to(torch.bfloat16).cuda()
    lengths = torch.tensor([t, max(t - 7, 0), min(t, 3), 0, t + 5], dtype=torch.int64).cuda()
    local_f32, top = local_topk(local, features, lengths)
    assert torch.equal(local_f32, local.float())
    ref = reference_top(local, features, lengths)
    assert torch.equal(torch.isnan(top), torch.isnan(ref))  # a clip without frames is NaN, as in the reference
    ok = ~torch.isnan(ref)
    torch.testing.assert_close(top[ok], ref[ok], rtol=1e-6, atol=1e-6)


def test_local_topk_ties_and_column_slices():
    """Scores on a coarse grid (many ties at the k-th value); features a function of
    the score, so every tie order gives one mean. Inputs are column slices of one
    [B, T, 264] buffer, as the decoder's single GEMM produces them."""
    gen = torch.Generator().manual_seed(11)
    b, t = 4, 300
    level = torch.randint(0, 13, (b, t), generator=gen)
    table = torch.randn(13, 256, generator=gen)
    both = torch.zeros(b, t, 264, dtype=torch.bfloat16)
    both[..., 0] = both[..., 1] = ((level.float() - 6) / 4).to(torch.bfloat16)
    both[..., 8:] = table[level].to(torch.bfloat16)
    both = both.cuda()
    lengths = torch.tensor([300, 100, 20, 1], dtype=torch.int64).cuda()
    local, features = both[..., :2], both[..., 8:]
    local_f32, top = local_topk(local, features, lengths)
    assert torch.equal(local_f32, local.float())
    torch.testing.assert_close(top, reference_top(local, features, lengths), rtol=1e-6, atol=1e-6)


def _heads_reference(dec, deep_h, fine_h, global_feature, memory, top):
    """decoder.py:77-89 under BF16 autocast, from the query-read rows."""
    deep_q = (deep_h[:, :4].mean(1), deep_h[:, 4:8].mean(1), deep_h[:, 8:].mean(1))
    fine_q = (fine_h[:, :4].mean(1), fine_h[:, 4:8].mean(1), fine_h[:, 8:].mean(1))
    with torch.autocast("cuda", dtype=torch.bfloat16):
        voice = dec.voice_lat(torch.cat((deep_q[0], fine_q[0], global_feature, top[:, 0], memory), -1))
        music = dec.music_lat(torch.cat((deep_q[1], fine_q[1], global_feature, top[:, 1], memory), -1))
        v, m = dec.voice_head(voice), dec.music_head(music)
        f = dec.file_head(torch.cat((deep_q[2], fine_q[2], global_feature, memory, voice, music), -1))
        return torch.cat((f, v[:, :1], m[:, :1], v[:, 1:], m[:, 1:]), -1).float()


@pytest.mark.parametrize("b", [1, 8, 13, 32])
def test_decoder_heads_against_autocast_layers(b):
    torch.manual_seed(b)
    dec = Decoder(384).cuda()
    with torch.no_grad():  # larger head weights than the default init, so the logits are not all near 0
        for layer in (dec.voice_head, dec.music_head, dec.file_head[2]):
            layer.weight.mul_(8)
    deep_h = torch.randn(b, 10, 256, device="cuda").to(torch.bfloat16)
    fine_h = torch.randn(b, 10, 256, device="cuda").to(torch.bfloat16)
    global_feature = torch.randn(b, 256, device="cuda").to(torch.bfloat16)
    memory = torch.randn(b, 256, device="cuda").to(torch.bfloat16)
    top = torch.randn(b, 2, 256, device="cuda")
    with torch.no_grad():
        ours = decoder_heads(deep_h, fine_h, global_feature, memory, top, dec)
        ref = _heads_reference(dec, deep_h, fine_h, global_feature, memory, top)
    assert ours.shape == (b, 5) and ours.dtype == torch.float32
    scale = ref.abs().max().item()
    assert (ours - ref).abs().max().item() <= 2 * scale / 128
    assert (ours == ref).float().mean().item() >= 0.6


def test_decoder_fused_tail_matches_pytorch_tail():
    """The decoder's forward with the fused tail against the same module's PyTorch tail
    (same native query reads and local GEMM, BF16 autocast), on one synthetic batch."""
    torch.manual_seed(3)
    dim, b, t, tf_ = 384, 6, 40, 90
    dec = Decoder(dim).cuda()
    dec.native_kernels = True
    x = torch.randn(b, t, dim, device="cuda")
    lengths = torch.tensor([40, 33, 12, 1, 40, 25], device="cuda")
    fine_lengths = torch.tensor([90, 70, 24, 3, 90, 50], device="cuda")
    fine = torch.randn(b, tf_, 8, 64, device="cuda").to(torch.bfloat16)
    mf = torch.randn(b, t, dim, device="cuda").to(torch.bfloat16)
    mb = torch.randn(b, t, dim, device="cuda").to(torch.bfloat16)
    grids = Grids.make(lengths, t, dim // 6, True, True)
    with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16):
        fused = dec(x, fine, grids, fine_lengths, mf, mb)
        dec.fused_tail = False
        plain = dec(x, fine, grids, fine_lengths, mf, mb)
    for key in ("local_logits", "local_mask", "features", "feature_mask", "embedding"):
        assert torch.equal(fused[key], plain[key]), key
    scale = plain["logits"].abs().max().item()
    assert (fused["logits"] - plain["logits"]).abs().max().item() <= 2 * scale / 128
