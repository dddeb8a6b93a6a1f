"""Text encoders of the served models, with the checkpoints' architectures and random weights.

* Wan2.1 / Wan2.2: UMT5-XXL encoder (d_model 4096, 24 layers, 64 heads x 64, gated-GELU FFN
  10240, 256 384-token vocabulary), 512 text tokens.
* SD3.5: CLIP-L/14 (768) and OpenCLIP bigG/14 (1280, with projection) text towers plus the
  T5-XXL v1.1 encoder (4096).  The joint context is the two CLIP penultimate hidden states
  concatenated on the feature axis, zero-padded to 4096 and stacked before the T5 tokens
  (77 + 256 = 333 tokens); the pooled vector is the two projected EOS embeddings (768 + 1280).

The layers are the ``transformers`` implementations (library code; the encoders run once per
request, off the denoising hot path) built from these configs, so a diffusers checkpoint's
``text_encoder*/`` weights load with ``load_state_dict``.  No tokenizer vocabularies ship
offline: ``HashTokenizer`` maps each whitespace word to a stable id (SHA-256) and appends EOS,
which keeps the token counts, the valid-token crop and the per-prompt determinism of the real
path.  Each encoder is a callable ``encode(prompt, max_len) -> (tokens [valid, dim], valid)``
for ``EncoderPool``; only the valid tokens are encoded (the reference's UMT5 valid-token crop,
identical to encoding the padded sequence under an attention mask).  Reference: the prompt
path of workers/ditserve/models/encoder_pool.py:41-471 and the SD3.5 pipeline's prompt
encoding (workers/ditserve/models/sd35.py).
"""
from __future__ import annotations

import hashlib

import torch

UMT5_XXL = dict(vocab_size=256384, d_model=4096, d_kv=64, d_ff=10240, num_layers=24, num_heads=64,
                relative_attention_num_buckets=32, relative_attention_max_distance=128,
                feed_forward_proj="gated-gelu", layer_norm_epsilon=1e-6)
T5_XXL = dict(vocab_size=32128, d_model=4096, d_kv=64, d_ff=10240, num_layers=24, num_heads=64,
              relative_attention_num_buckets=32, relative_attention_max_distance=128,
              feed_forward_proj="gated-gelu", layer_norm_epsilon=1e-6)
CLIP_L = dict(vocab_size=49408, hidden_size=768, intermediate_size=3072, num_hidden_layers=12,
              num_attention_heads=12, max_position_embeddings=77, projection_dim=768, hidden_act="quick_gelu")
CLIP_G = dict(vocab_size=49408, hidden_size=1280, intermediate_size=5120, num_hidden_layers=32,
              num_attention_heads=20, max_position_embeddings=77, projection_dim=1280, hidden_act="gelu")
# test-sized stand-ins with the same structure
TINY_T5 = dict(vocab_size=1000, d_model=64, d_kv=16, d_ff=128, num_layers=2, num_heads=4,
               relative_attention_num_buckets=32, relative_attention_max_distance=128,
               feed_forward_proj="gated-gelu", layer_norm_epsilon=1e-6)
TINY_CLIP_L = dict(vocab_size=1000, hidden_size=16, intermediate_size=32, num_hidden_layers=2,
                   num_attention_heads=4, max_position_embeddings=77, projection_dim=16, hidden_act="quick_gelu")
TINY_CLIP_G = dict(vocab_size=1000, hidden_size=32, intermediate_size=64, num_hidden_layers=2,
                   num_attention_heads=4, max_position_embeddings=77, projection_dim=32, hidden_act="gelu")


class HashTokenizer:
    """Stable word -> id map in [first_id, vocab - 1), EOS = vocab - 1 (also the largest id)."""

    def __init__(self, vocab_size: int, first_id: int = 2, bos: int | None = None):
        self.vocab, self.first, self.bos = int(vocab_size), int(first_id), bos
        self.eos = self.vocab - 1

    def __call__(self, text: str, max_len: int) -> list[int]:
        ids = [] if self.bos is None else [self.bos]
        for w in text.split():
            h = int(hashlib.sha256(w.encode()).hexdigest()[:12], 16)
            ids.append(self.first + h % (self.vocab - 1 - self.first))
        return ids[:max_len - 1] + [self.eos]


def _init(model: torch.nn.Module, seed: int, device, dtype):
    """Seeded weights: N(0, 0.02) matrices and embeddings, unit norm gains, zero biases."""
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in sorted(model.named_parameters()):
            if p.dim() > 1:
                p.copy_(torch.randn(p.shape, generator=g) * 0.02)
            elif name.endswith("bias"):
                p.zero_()
            else:
                p.fill_(1.0)
    return model.to(device=device, dtype=dtype).eval()


class UMT5TextEncoder:
    """Wan's text encoder: ``(prompt, max_len) -> ([valid, d_model], valid)``."""

    def __init__(self, config: dict | None = None, device="cpu", dtype=torch.float32, seed: int = 0, t5: bool = False):
        from transformers import T5Config, T5EncoderModel, UMT5Config, UMT5EncoderModel
        cfg = dict(config or (T5_XXL if t5 else UMT5_XXL))
        cls_cfg, cls = (T5Config, T5EncoderModel) if t5 else (UMT5Config, UMT5EncoderModel)
        self.model = _init(cls(cls_cfg(**cfg)), seed, device, dtype)
        self.tok = HashTokenizer(cfg["vocab_size"])
        self.dim, self.device = cfg["d_model"], device

    @torch.inference_mode()
    def __call__(self, prompt: str, max_len: int):
        ids = torch.tensor([self.tok(prompt, max_len)], device=self.device)
        out = self.model(input_ids=ids).last_hidden_state[0]
        return out.float().cpu(), ids.shape[1]


class SD3TextEncoders:
    """CLIP-L + CLIP-G + T5-XXL: ``encode(prompt) -> (context [77 + t5_len, 4096], pooled [2048])``."""

    def __init__(self, tiny: bool = False, device="cpu", dtype=torch.float32, seed: int = 0, t5_len: int = 256,
                 tiny_dims: tuple[int, int, int] | None = None):
        """``tiny_dims`` = (CLIP-L width, CLIP-G width, T5 width) of a test-sized set."""
        from transformers import CLIPTextConfig, CLIPTextModelWithProjection
        lcfg, gcfg = (TINY_CLIP_L, TINY_CLIP_G) if tiny else (CLIP_L, CLIP_G)
        t5cfg = TINY_T5 if tiny else T5_XXL
        if tiny and tiny_dims is not None:
            wl, wg, wt = tiny_dims
            lcfg = dict(lcfg, hidden_size=wl, intermediate_size=2 * wl, projection_dim=wl)
            gcfg = dict(gcfg, hidden_size=wg, intermediate_size=2 * wg, projection_dim=wg)
            t5cfg = dict(t5cfg, d_model=wt, d_kv=wt // t5cfg["num_heads"], d_ff=2 * wt)
        self.clip_l = _init(CLIPTextModelWithProjection(CLIPTextConfig(**lcfg, eos_token_id=lcfg["vocab_size"] - 1)),
                            seed, device, dtype)
        self.clip_g = _init(CLIPTextModelWithProjection(CLIPTextConfig(**gcfg, eos_token_id=gcfg["vocab_size"] - 1)),
                            seed + 1, device, dtype)
        self.t5 = UMT5TextEncoder(t5cfg, device, dtype, seed + 2, t5=True)
        self.clip_tok = HashTokenizer(lcfg["vocab_size"], bos=lcfg["vocab_size"] - 2)
        self.t5_len, self.device = t5_len, device
        self.joint_dim = self.t5.dim
        self.pooled_dim = lcfg["projection_dim"] + gcfg["projection_dim"]

    @torch.inference_mode()
    def __call__(self, prompt: str):
        ids = self.clip_tok(prompt, 77)
        ids = ids + [ids[-1]] * (77 - len(ids))  # CLIP pads with EOS to its 77 positions
        x = torch.tensor([ids], device=self.device)
        hs, pooled = [], []
        for enc in (self.clip_l, self.clip_g):
            o = enc(input_ids=x, output_hidden_states=True)
            hs.append(o.hidden_states[-2][0].float())  # penultimate layer
            pooled.append(o.text_embeds[0].float())
        clip = torch.cat(hs, dim=-1)
        if clip.shape[-1] > self.joint_dim:
            raise ValueError("the CLIP features are wider than the T5 width")
        clip = torch.nn.functional.pad(clip, (0, self.joint_dim - clip.shape[-1]))
        t5, valid = self.t5(prompt, self.t5_len)
        t5 = torch.nn.functional.pad(t5, (0, 0, 0, self.t5_len - valid))  # zero rows past the valid tokens
        return torch.cat([clip.cpu(), t5], dim=0), torch.cat(pooled).cpu()
