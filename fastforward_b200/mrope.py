"""Host-side interleaved M-RoPE tables for one request geometry (computed once per key).

The reference precomputes the 3-axis position ids per (side, bucket) on the host with
the model's `get_rope_index` (`scaled_qwen_runtime.py:83-96`, `_family/depth_runtime.py:
160-177`) and evaluates `rotary_emb` per replay; here both are evaluated once per graph
key on the host in fp32 and uploaded as bf16 [T, 128] cos/sin tables.

Positions (Qwen3-VL, spatial merge 2): text before the image counts 0..s-1 on all axes;
image token (row r, col c) of the gh x gw merged grid gets (t, h, w) = (s, s + r, s + c);
text after the image (bucket padding included) resumes at s + max(gh, gw).
Frequencies: inv_freq[i] = theta^(-2i/128); frequency i uses the H axis when i % 3 == 1
and i < 3*sections[1], the W axis when i % 3 == 2 and i < 3*sections[2], else T;
emb = cat(f, f); cos/sin evaluated in fp32 and rounded to bf16.
"""
import torch


def position_ids(n_tokens, image_start, grid_h, grid_w, merge=2):
    gh, gw = grid_h // merge, grid_w // merge
    nv = gh * gw
    if image_start + nv > n_tokens:
        raise ValueError(f"image window [{image_start}, {image_start + nv}) exceeds {n_tokens} tokens")
    pos = torch.empty(3, n_tokens, dtype=torch.long)
    pos[:, :image_start] = torch.arange(image_start)
    s = image_start
    pos[0, s:s + nv] = s
    pos[1, s:s + nv] = s + torch.arange(gh).repeat_interleave(gw)
    pos[2, s:s + nv] = s + torch.arange(gw).repeat(gh)
    rest = n_tokens - (s + nv)
    pos[:, s + nv:] = s + max(gh, gw) + torch.arange(rest)
    return pos


def cos_sin(pos, head_dim=128, theta=5_000_000.0, sections=(24, 20, 20)):
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    freqs = pos.float()[:, :, None] * inv_freq[None, None, :]
    f = freqs[0].clone()
    for axis in (1, 2):
        idx = torch.arange(axis, sections[axis] * 3, 3)
        f[:, idx] = freqs[axis][:, idx]
    emb = torch.cat((f, f), -1)  # equal halves: the fused qkv epilogue reads columns [0, 64) only
    return emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
