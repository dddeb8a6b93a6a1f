"""Text encoders with the checkpoints' architectures (test-sized configs, random weights):
the valid-token crop equals masked encoding of the padded sequence, SD3 joint conditioning has
the pipeline's layout, and both plug into the encoder pool."""
import torch

from ditserve_b200.models.encoder_pool import EncoderPool
from ditserve_b200.models.text_encoders import (TINY_T5, HashTokenizer, SD3TextEncoders, UMT5TextEncoder,
                                                UMT5_XXL)


def test_hash_tokenizer_is_stable_and_bounded():
    tok = HashTokenizer(1000)
    a = tok("a red fox jumps", 16)
    assert a == tok("a red fox jumps", 16) and a[-1] == 999 and len(a) == 5
    assert all(2 <= i < 999 for i in a[:-1])
    assert len(tok(" ".join(["w"] * 40), 16)) == 16


def test_umt5_valid_token_crop_equals_masked_padding():
    enc = UMT5TextEncoder(TINY_T5, seed=3)
    out, valid = enc("a cat on a red sofa", 32)
    assert out.shape == (valid, 64) and valid == 7
    ids = torch.tensor([enc.tok("a cat on a red sofa", 32) + [0] * (32 - valid)])
    mask = torch.zeros(1, 32, dtype=torch.long)
    mask[0, :valid] = 1
    with torch.no_grad():
        full = enc.model(input_ids=ids, attention_mask=mask).last_hidden_state[0, :valid]
    torch.testing.assert_close(out, full, rtol=1e-5, atol=1e-5)
    assert UMT5_XXL["d_model"] == 4096 and UMT5_XXL["vocab_size"] == 256384


def test_sd3_joint_conditioning_layout():
    enc = SD3TextEncoders(tiny=True, t5_len=16)
    ctx, pooled = enc("a lighthouse at dusk")
    assert ctx.shape == (77 + 16, 64) and pooled.shape == (16 + 32,)
    assert torch.count_nonzero(ctx[:77, 48:]) == 0           # CLIP features zero-padded to the T5 width
    assert torch.count_nonzero(ctx[:77, :48]) > 0
    assert torch.count_nonzero(ctx[77 + 5:]) == 0          # T5 rows past the valid tokens are zero
    assert torch.count_nonzero(ctx[77:77 + 5]) > 0
    ctx2, pooled2 = enc("a lighthouse at dusk")
    assert torch.equal(ctx, ctx2) and torch.equal(pooled, pooled2)


def test_encoder_pool_with_umt5(tmp_path):
    enc = UMT5TextEncoder(TINY_T5, seed=1)
    pool = EncoderPool(enc, max_len=24, slab_dir=str(tmp_path))
    try:
        t = pool.submit("a small boat", negative="blurry")
        got = pool.fetch(t, dtype=torch.float32)
        assert got is not None
    finally:
        pool.close()


def test_wan_backend_encodes_prompts_with_umt5(tmp_path):
    from ditserve_b200.models.wan.backend import WanBackend
    w = WanBackend({"model": "wan-tiny", "device": "cpu", "transfer_dir": str(tmp_path),
                    "text_encoder": {"config": "tiny", "seed": 4}})
    base = dict(height=32, width=32, frames=5, steps=2, seed=3, guidance=4.0, negative_prompt="blurry")
    outs = {}
    for sid, prompt in (("a", "a red fox in snow"), ("b", "a red fox in snow"), ("c", "a blue whale")):
        w.prepare(dict(id=1, spec=dict(base, request_id=sid, prompt=prompt)))
        st = w.states[sid]
        assert st.context.shape == (1, 16, 64) and torch.count_nonzero(st.context[0, 6:]) == 0
        w.advance(dict(id=2, state_id=sid, steps=2))
        outs[sid] = w.finish(dict(id=3, state_id=sid, output_mode="digest"))["value"]
    assert outs["a"] == outs["b"] and outs["a"] != outs["c"]


def test_sd35_backend_encodes_prompts_with_clip_and_t5():
    from ditserve_b200.models.sd35.backend import SD35Backend
    b = SD35Backend({"model": "sd3.5-tiny", "device": "cpu", "text_encoder": {"config": "tiny", "seed": 2}})
    spec = dict(height=64, width=64, steps=2, seed=1, guidance=3.0, text_len=90, negative_prompt="low quality")
    outs = {}
    for sid, prompt in (("a", "a teapot"), ("b", "a teapot"), ("c", "a castle")):
        b.prepare(dict(id=1, spec=dict(spec, request_id=sid, prompt=prompt)))
        st = b.states[sid]
        assert st.context.shape == (90, 256) and st.pooled.shape == (128,)
        while not st.done:
            b.engine.advance_batch([st])
        outs[sid] = st.latents.clone()
    assert torch.equal(outs["a"], outs["b"]) and not torch.equal(outs["a"], outs["c"])
