"""Batched prefill (sx_prefill_batch) on a B200 against the CPU checker's token-by-token decode.

The reference prefills a prompt with one forwardToken per token (src/model/forward.zig:19-75);
the checker does exactly that per session, with its bf16 projection mode on: the tensor-core
path multiplies bf16 operands -- the normed residual, the attention output and the GeGLU
product rounded to bf16, and each dequantised weight (f32)(nib - 8) * d rounded to bf16 (the
operand the GEMM dequantises into shared memory, bit-exact per the dequant tests) -- and the
checker rounds the same values.  Where the two round different f32 values that straddle a
bf16 boundary, one operand differs by 2^-8 (double rounding); logits are therefore compared
with conftest.assert_close_bf16_operands (the f32 tolerance on all but 1% of elements,
every element within 1e-3 of the logit scale); greedy tokens with the top-2 margin rule; the
caches the prefill wrote are checked by decoding on from them (checker back in f32 mode).  The KV cache
is f32 here for the reason given in test_gpu_batch.py."""
import numpy as np
import pytest

import sx
from oracle import oracle as orc
from tests.conftest import BF16_KV_FRAC
from tests.conftest import assert_close_bf16_operands as assert_close
from tests.test_gpu_model import margin_top2, tiny_cfg

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")


def prompts_for(cfg, seed, lens):
    rng = np.random.default_rng(seed)
    H = cfg["hidden_size"]
    ids = [rng.integers(0, cfg["vocab_size"], n) for n in lens]
    return [np.stack([sx.synth_embed_row(H, int(t), seed) for t in row]) for row in ids]


def checker_prefill(cfg, seed, prompt, start=0, ref=None):
    ref = ref or orc.Model(cfg, seed)
    ref.set_act_bf16(True)
    n = len(prompt)
    for j in range(n):
        tok, lg, _ = ref.forward(prompt[j], start + j, j == n - 1)
    ref.set_act_bf16(False)
    return ref, tok, lg


def check_token(tok, rtok, rlg, what):
    if tok != rtok:
        assert margin_top2(rlg) < 1e-3, f"{what}: token {tok} vs {rtok}"


@pytest.mark.parametrize("lens", [[5, 12, 9], [1, 7, 12]])
def test_prefill_matches_checker_then_decodes_on(engine_f32kv, lens):
    engine = engine_f32kv
    cfg = tiny_cfg(num_sessions=3, num_layers=3, kv_bf16=0)
    seed = 31
    model = sx.Model(engine, sx.model_config(**cfg))
    model.synth_weights(seed)
    prompts = prompts_for(cfg, seed, lens)
    rings = [sx.Ring(1, cfg["num_anchors"], cfg["window_size"], cfg["num_recall"]) for _ in lens]
    logits = np.zeros((len(lens), cfg["vocab_size"]), np.float32)
    toks = model.prefill_batch(prompts, rings, [0] * len(lens), logits_out=logits)
    refs = []
    for s, p in enumerate(prompts):
        ref, rtok, rlg = checker_prefill(cfg, seed, p)
        assert_close(logits[s], rlg, what=f"session {s} prefill logits")
        check_token(int(toks[s]), rtok, rlg, f"session {s} prefill")
        refs.append(ref)
    # decode on from the caches the prefill wrote (batch step over the three sessions)
    clocks = list(lens)
    tokens = [int(t) for t in toks]
    for step in range(3):
        xs = np.stack([sx.synth_embed_row(cfg["hidden_size"], tokens[s], seed) for s in range(3)])
        slots = [rings[s].activate_slot(0, clocks[s]) for s in range(3)]
        lists = [rings[s].get_active_slots(0, clocks[s]) for s in range(3)]
        lg = np.zeros((3, cfg["vocab_size"]), np.float32)
        got = model.decode_batch(xs, clocks, slots, lists, True, lg)
        for s in range(3):
            rtok, rlg, _ = refs[s].forward(xs[s], clocks[s], True)
            assert_close(lg[s], rlg, what=f"session {s} decode step {step}")
            check_token(int(got[s]), rtok, rlg, f"session {s} decode step {step}")
            tokens[s] = int(got[s])
        clocks = [c + 1 for c in clocks]


def test_prefill_one_session_model_12b_width_head(engine_f32kv):
    # one-session model, 12B hidden / head widths, two layers, full vocabulary
    cfg = tiny_cfg(vocab_size=262144, hidden_size=3840, intermediate_size=15360, num_layers=2,
                   num_q_heads=16, num_kv_heads=8, num_global_kv_heads=8, head_dim=256,
                   global_head_dim=256, num_anchors=32, window_size=512, num_recall=96,
                   full_every=2, kv_bf16=0)
    seed = 5
    model = sx.Model(engine_f32kv, sx.model_config(**cfg))
    model.synth_weights(seed)
    (prompt,) = prompts_for(cfg, seed, [40])
    ring = sx.Ring(1, cfg["num_anchors"], cfg["window_size"], cfg["num_recall"])
    logits = np.zeros((1, cfg["vocab_size"]), np.float32)
    (tok,) = model.prefill_batch([prompt], [ring], [0], logits_out=logits)
    ref, rtok, rlg = checker_prefill(cfg, seed, prompt)
    assert_close(logits[0], rlg, what="12B-width prefill logits")
    check_token(int(tok), rtok, rlg, "12B-width prefill")
    # and one decode step through sx_forward_token on the prefilled cache
    x = sx.synth_embed_row(cfg["hidden_size"], int(tok), seed)
    slot = ring.activate_slot(0, 40)
    lg1 = np.zeros(cfg["vocab_size"], np.float32)
    t1 = model.forward_token(x, 40, slot, ring.get_active_slots(0, 40), True, lg1)
    r1, rl1, _ = ref.forward(x, 40, True)
    assert_close(lg1, rl1, what="decode after prefill")
    check_token(t1, r1, rl1, "decode after prefill")


def test_prompt_longer_than_the_window_is_split(engine_f32kv):
    engine = engine_f32kv
    cfg = tiny_cfg(num_sessions=1, num_layers=2, kv_bf16=0)
    seed = 12
    model = sx.Model(engine, sx.model_config(**cfg))
    model.synth_weights(seed)
    (prompt,) = prompts_for(cfg, seed, [15])  # clock 12 rewrites slot 4 (window of 8 after 4)
    ring = sx.Ring(1, cfg["num_anchors"], cfg["window_size"], cfg["num_recall"])
    with pytest.raises(sx.SxError):
        model.prefill_batch([prompt], [ring], [0])
    ring = sx.Ring(1, cfg["num_anchors"], cfg["window_size"], cfg["num_recall"])
    wrapped = sx.Ring(1, 4, 8, 4)
    wrapped.prefill(0, 12)  # the ring after clocks 0..11
    with pytest.raises(sx.SxError):  # token 12 lists slot 5, which token 13 rewrites
        model.prefill_batch([prompt[12:]], [wrapped], [12])
    model.prefill_batch([prompt[:12]], [ring], [0])
    # once the window has wrapped, every token rewrites a slot the one before it reads
    logits = np.zeros((1, cfg["vocab_size"]), np.float32)
    for j in (12, 13, 14):
        (tok,) = model.prefill_batch([prompt[j:j + 1]], [ring], [j], logits_out=logits)
    ref, rtok, rlg = checker_prefill(cfg, seed, prompt)
    assert_close(logits[0], rlg, what="split prefill logits")
    check_token(int(tok), rtok, rlg, "split prefill")


def test_prefill_rejects_bad_tokens(engine):
    cfg = tiny_cfg(num_sessions=2, num_layers=1)
    model = sx.Model(engine, sx.model_config(**cfg))
    (p,) = prompts_for(cfg, 1, [3])
    rings = [sx.Ring(1, 4, 8, 4)]
    with pytest.raises(sx.SxError):
        model.prefill_batch([p], rings, [0], sessions=[2])  # session beyond the model's two


@pytest.mark.parametrize("head_dim,nq,nkv", [(256, 8, 1), (256, 4, 2), (256, 2, 2), (128, 4, 2),
                                             (64, 4, 2)])
def test_prefill_bf16_kv_matches_checker(engine, head_dim, nq, nkv):
    """The bf16-KV prefill attention against the checker in its bf16-cache, bf16-operand mode:
    head_dim 256 runs the tensor-core kernel (8, 2 and 1 q heads per kv head: 8, 32 and 64
    tokens per work item), 128 and 64 the CUDA-core kernel's 4- and 2-element cached-row loads."""
    cfg = tiny_cfg(num_sessions=3, num_layers=3, kv_bf16=1, head_dim=head_dim,
                   global_head_dim=head_dim, num_q_heads=nq, num_kv_heads=nkv,
                   num_global_kv_heads=nkv, hidden_size=512, intermediate_size=1024)
    seed = 41
    model = sx.Model(engine, sx.model_config(**cfg))
    model.synth_weights(seed)
    lens = [11, 3, 12]
    prompts = prompts_for(cfg, seed, lens)
    rings = [sx.Ring(1, cfg["num_anchors"], cfg["window_size"], cfg["num_recall"]) for _ in lens]
    logits = np.zeros((3, cfg["vocab_size"]), np.float32)
    toks = model.prefill_batch(prompts, rings, [0] * 3, logits_out=logits)
    for s, p in enumerate(prompts):
        _, rtok, rlg = checker_prefill(cfg, seed, p)
        assert_close(logits[s], rlg, what=f"session {s} prefill logits", frac=BF16_KV_FRAC)
        check_token(int(toks[s]), rtok, rlg, f"session {s} prefill")


def test_config5_shape_ragged_prefill_bf16_kv_then_batch8_decode(engine):
    """Config 5 as bench.py --case sessions runs it (bf16 cache, 8 q heads per kv head, full
    vocabulary), on ragged prompts of 8 sessions and fewer layers: the batched prefill against
    the checker's token-by-token decode (bf16 operands, bf16 cache), then two batch-8 decode
    steps from the caches the prefill wrote."""
    from tests.test_gpu_batch import c5_cfg
    cfg = c5_cfg(num_layers=5)
    seed = 77
    model = sx.Model(engine, sx.model_config(**cfg))
    model.synth_weights(seed)
    lens = [16, 40, 7, 64, 23, 1, 50, 33]
    prompts = prompts_for(cfg, seed, lens)
    rings = [sx.Ring(1, cfg["num_anchors"], cfg["window_size"], cfg["num_recall"]) for _ in lens]
    logits = np.zeros((8, cfg["vocab_size"]), np.float32)
    toks = model.prefill_batch(prompts, rings, [0] * 8, logits_out=logits)
    refs = []
    for s, p in enumerate(prompts):
        ref, rtok, rlg = checker_prefill(cfg, seed, p)
        assert_close(logits[s], rlg, what=f"session {s} prefill logits", frac=BF16_KV_FRAC)
        check_token(int(toks[s]), rtok, rlg, f"session {s} prefill")
        refs.append(ref)
    clocks, tokens = list(lens), [int(t) for t in toks]
    for step in range(2):
        xs = np.stack([sx.synth_embed_row(cfg["hidden_size"], tokens[s], seed) for s in range(8)])
        slots = [rings[s].activate_slot(0, clocks[s]) for s in range(8)]
        lists = [rings[s].get_active_slots(0, clocks[s]) for s in range(8)]
        lg = np.zeros((8, cfg["vocab_size"]), np.float32)
        got = model.decode_batch(xs, clocks, slots, lists, True, lg)
        for s in range(8):
            rtok, rlg, _ = refs[s].forward(xs[s], clocks[s], True)
            assert_close(lg[s], rlg, what=f"session {s} decode step {step}", frac=BF16_KV_FRAC)
            check_token(int(got[s]), rtok, rlg, f"session {s} decode step {step}")
            tokens[s] = int(got[s])
        clocks = [c + 1 for c in clocks]


def test_long_prompts_tensor_core_attention_spans_several_key_tiles(engine):
    """Prompts of 300 and 181 tokens on config 5's head shape (one kv head, 8 q heads, 640-slot
    ring): each work item's key union covers several 64-key tiles, so the online softmax runs
    across tiles and the last tile is partly empty; against the checker."""
    from tests.test_gpu_batch import c5_cfg
    cfg = c5_cfg(num_layers=2, num_sessions=2)
    seed = 91
    model = sx.Model(engine, sx.model_config(**cfg))
    model.synth_weights(seed)
    lens = [300, 181]
    prompts = prompts_for(cfg, seed, lens)
    rings = [sx.Ring(1, cfg["num_anchors"], cfg["window_size"], cfg["num_recall"]) for _ in lens]
    logits = np.zeros((2, cfg["vocab_size"]), np.float32)
    toks = model.prefill_batch(prompts, rings, [0] * 2, logits_out=logits)
    for s, p in enumerate(prompts):
        _, rtok, rlg = checker_prefill(cfg, seed, p)
        assert_close(logits[s], rlg, what=f"session {s} prefill logits", frac=BF16_KV_FRAC)
        check_token(int(toks[s]), rtok, rlg, f"session {s} prefill")
