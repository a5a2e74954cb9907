"""Model-level parity of the device model (include/q38cuda_model.h) with the
upstream Q38Model compiled from its sources, on one seeded synthetic GGUF that
has the upstream loader's exact tensor names, shapes and metadata, the
Q4_K_M-style type mix and well-conditioned weights (q38b200.gguf, dist
"conditioned").

Why the full-model bar is relative to the upstream itself.  Every projection
input is re-quantized to Q8_K, so a one-ulp difference anywhere (a different
but legal summation order, a libm expf that differs from glibc's in the last
bit) flips a few int8 activations, and the flips random-walk through the 64
layers up to the Q8_K noise floor.  The upstream's own native (AVX2) and
portable C builds drift apart exactly this way (on the real checkpoint RMSE
0.058 on logits near 25, docs/CORRECTNESS.md of the upstream; on this synthetic
model their top-1 differs on several tokens).  So:

* every layer is checked with teacher forcing, with its recurrent state and KV
  cache, over several tokens: the device's own input to layer L goes through
  the CPU restatement (oracle/model_oracle.py, with the upstream's Q8_K
  kernels) and must match the device's layer output to rounding (1e-5) except
  for rare in-layer int8 flips (1e-2);
* the first layer, whose input is exact, must match the upstream model to 1e-5;
* over a token sequence the device's logits may not drift from the native
  upstream build further than the upstream's portable build does (with 50 %
  slack), and top-1 must agree wherever the native top-2 margin is above 5 %
  of the top logit;
* the device's own paths must agree bit for bit: prefill vs token-by-token
  decode, the device-side greedy loop vs step-by-step argmax, and speculative
  decoding vs plain greedy decoding.
"""
import numpy as np
import pytest

import oracle as O
from q38b200 import gguf

pytestmark = pytest.mark.gpu

COSINE = 0.999
MARGIN = 0.05


@pytest.fixture(scope="module")
def model_path():
    return gguf.cached_model_path(seed=1, mtp=True, dist="conditioned")


@pytest.fixture(scope="module")
def portable(model_path):
    if not __import__("os").path.exists(O.REF_PORTABLE_LIB):
        pytest.skip("portable upstream build missing")
    ref = O.ReferenceModel(model_path, 512, lib_path=O.REF_PORTABLE_LIB)
    yield ref
    ref.close()


@pytest.fixture(scope="module")
def models(model_path):
    if not O.reference_available():
        pytest.skip("upstream reference library not built")
    from q38b200.model import Model
    dev = Model(model_path, 512)
    ref = O.ReferenceModel(model_path, 512)
    yield dev, ref
    dev.close()
    ref.close()


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / np.linalg.norm(b)


def cosine(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return a @ b / np.linalg.norm(a) / np.linalg.norm(b)


def safe_margin(logits):
    s = np.sort(logits)
    return (s[-1] - s[-2]) >= MARGIN * abs(s[-1])


def check_logits(got, want, what, cos_min=COSINE, top1=True):
    assert np.all(np.isfinite(got)), what
    c = cosine(got, want)
    assert c >= cos_min, f"{what}: cosine {c:.6f}"
    if top1 and safe_margin(want):
        assert int(np.argmax(got)) == int(np.argmax(want)), f"{what}: top-1 differs at a safe margin"


def test_first_layer_matches_upstream(models):
    """Layer 0 sees the exact embedding row, so only in-layer rounding separates
    the two (observed ~7e-7)."""
    dev, ref = models
    for token in (777, 3):
        dev.reset()
        ref.reset()
        assert rel(dev.forward_token_layers(token, 1), ref.forward_token_layers(token, 1)) <= 1e-5


def test_layers_teacher_forced(models, model_path):
    """Each layer, with its state, over 3 tokens (positions 0..2).  At least
    85 % of the (layer, token) outputs must match to rounding: the DeltaNet
    beta/alpha rows are float-path Q8_0 dot products that the upstream sums in
    one 5120-step sequential fmaf chain (qwen38_quant.c:496-508) and the
    device sums in parallel, so a few more outputs than the other layers'
    rounding alone would give see an int8 flip of a later Q8_K activation."""
    import model_oracle as MO
    dev, _ = models
    lo = MO.LayerOracle(model_path, O.Reference())
    tokens = (4321, 17, 99999)
    errors = []
    for layer in range(64):
        dev.reset()
        inputs = [dev.forward_token_layers(t, layer) for t in tokens]
        dev.reset()
        outputs = [dev.forward_token_layers(t, layer + 1) for t in tokens]
        sl = MO.StatefulLayer(lo, layer)
        errors += [rel(o, sl.step(i)) for i, o in zip(inputs, outputs)]
    errors = np.array(errors)
    assert errors.max() <= 1e-2, f"worst (layer, token) {divmod(int(errors.argmax()), 3)}: {errors.max():.2e}"
    exact = np.mean(errors <= 1e-5)
    assert exact >= 0.85, f"{exact:.3f} exact; off: {[divmod(int(i), 3) for i in np.nonzero(errors > 1e-5)[0]]}"


def test_attention_layer_long_context_teacher_forced(models, model_path):
    """The first full-attention layer (3), teacher-forced over 150 positions:
    the device splits a token's positions over 1, 2 and then 3 CTAs of its
    cluster (one per 64 positions) and merges them in rank order, which must
    stay within rounding of the upstream single-pass softmax."""
    import model_oracle as MO
    dev, _ = models
    lo = MO.LayerOracle(model_path, O.Reference())
    layer = 3
    tokens = np.random.default_rng(21).integers(0, 248320, 150).tolist()
    dev.reset()
    inputs = [dev.forward_token_layers(t, layer) for t in tokens]
    dev.reset()
    outputs = [dev.forward_token_layers(t, layer + 1) for t in tokens]
    sl = MO.StatefulLayer(lo, layer)
    errors = np.array([rel(o, sl.step(i)) for i, o in zip(inputs, outputs)])
    # Positions either match to rounding or differ by a few int8 flips of a
    # Q8_K activation (~3e-3).  The oracle's softmax runs in float64 and the
    # device's in float32, so flips grow more frequent with the number of
    # positions (whatever the CTA count): the multi-CTA positions (64 and up)
    # are held to a majority of exact matches, not to the short ones' rate.
    exact_single, exact_multi = np.mean(errors[:64] <= 1e-5), np.mean(errors[64:] <= 1e-5)
    stats = f"exact {exact_single:.2f} (1 CTA) / {exact_multi:.2f} (2-3 CTAs), worst {errors.max():.2e}"
    assert errors.max() <= 1e-2, stats
    assert np.median(errors) <= 1e-5 and exact_single >= 0.8 and exact_multi >= 0.6, stats


def test_fp16_kv_cache_attention_layer_teacher_forced(model_path):
    """The optional fp16 KV cache (Q38CU_KV_F16=1 at open; the upstream keeps
    fp32, qwen38_model.c:1391-1396): the first full-attention layer, teacher-
    forced over 150 positions, stays within the in-layer int8-flip bar of the
    CPU restatement (fp16 keys and values round at 2^-11: measured median
    3.3e-3, worst 4.7e-3 against 1e-5 with the fp32 cache), and the 8-token
    prefill still equals token-by-token decoding bit for bit."""
    import os
    import model_oracle as MO
    from q38b200.model import Model
    if not O.reference_available():
        pytest.skip("upstream reference library not built")
    os.environ["Q38CU_KV_F16"] = "1"
    try:
        dev = Model(model_path, 512)
    finally:
        del os.environ["Q38CU_KV_F16"]
    try:
        lo = MO.LayerOracle(model_path, O.Reference())
        layer = 3
        tokens = np.random.default_rng(21).integers(0, 248320, 150).tolist()
        dev.reset()
        inputs = [dev.forward_token_layers(t, layer) for t in tokens]
        dev.reset()
        outputs = [dev.forward_token_layers(t, layer + 1) for t in tokens]
        sl = MO.StatefulLayer(lo, layer)
        errors = np.array([rel(o, sl.step(i)) for i, o in zip(inputs, outputs)])
        print(f"fp16 KV, attention layer teacher-forced: median {np.median(errors):.2e}, worst {errors.max():.2e}")
        assert errors.max() <= 1e-2 and np.median(errors) <= 5e-3
        prompt = np.random.default_rng(5).integers(0, 248320, 11).tolist()
        dev.reset()
        stepwise = [dev.forward_token(t) for t in prompt][-1]
        dev.reset()
        assert np.array_equal(dev.prefill(prompt), stepwise)
    finally:
        dev.close()


def test_forward_token_drift_within_upstream_builds(models, portable):
    dev, ref = models
    for m in (dev, ref, portable):
        m.reset()
    dev_err, port_err = [], []
    for token in (11, 2222, 33333, 5, 200000, 77):
        want = ref.forward_token(token)
        got, alt = dev.forward_token(token), portable.forward_token(token)
        assert np.all(np.isfinite(got))
        dev_err.append(rel(got, want))
        port_err.append(rel(alt, want))
        if safe_margin(want):
            assert int(np.argmax(got)) == int(np.argmax(want)), f"token {token}: top-1 differs at a safe margin"
    assert dev.position == ref.position == 6
    assert np.mean(dev_err) <= 1.5 * np.mean(port_err) + 1e-3, (dev_err, port_err)


def test_prefill_matches_decode_bitwise_and_upstream(models):
    dev, ref = models
    prompt = np.random.default_rng(5).integers(0, 248320, 11).tolist()  # one chunk of 8, one of 3
    dev.reset()
    stepwise = [dev.forward_token(t) for t in prompt][-1]
    dev.reset()
    batched = dev.prefill(prompt)
    assert np.array_equal(batched, stepwise), "prefill and token-by-token decode must agree bit for bit"
    assert dev.position == 11
    ref.reset()
    check_logits(batched, ref.prefill(prompt), "prefill", cos_min=0.9)
    # decoding continues from the prefilled state
    check_logits(dev.forward_token(42), ref.forward_token(42), "decode after prefill", cos_min=0.9)


def test_tensor_core_prefill_matches_upstream(models):
    """A 72-token prompt takes the tensor-core layer-major prefill (every
    projection one tcgen05 GEMM over the prompt, fp16 operands).  Its
    last-token logits may differ from the upstream prefill no more than the
    device's integer path (8-token chunks, bit-exact kernels) does, plus the
    fp16 rounding (50 % slack and 1e-3); top-1 must agree at a safe margin;
    decoding continues from the prefilled state."""
    import os
    dev, ref = models
    prompt = np.random.default_rng(72).integers(0, 248320, 72).tolist()
    os.environ["Q38CU_TC_PREFILL"] = "0"
    try:
        dev.reset()
        integer = dev.prefill(prompt)
    finally:
        del os.environ["Q38CU_TC_PREFILL"]
    dev.reset()
    tc = dev.prefill(prompt)
    assert dev.position == 72
    ref.reset()
    want = ref.prefill(prompt)
    check_logits(tc, want, "tensor-core prefill", cos_min=0.9)
    e_tc, e_int = rel(tc, want), rel(integer, want)
    print(f"prefill relative error vs upstream: tensor cores {e_tc:.3e}, integer path {e_int:.3e}")
    assert e_tc <= 1.5 * e_int + 1e-3, (e_tc, e_int)
    check_logits(dev.forward_token(42), ref.forward_token(42), "decode after tensor-core prefill", cos_min=0.9)


def test_tensor_core_prefill_continues_a_cached_prefix(models):
    """A second tensor-core prefill on top of a first (positions 70 .. 199,
    ragged 64-token tiles): attention reads the keys and values the first one
    cached, the DeltaNet conv window reads the ring and the state carries
    over.  Same bar as a single prefill against the upstream doing the same."""
    import os
    dev, ref = models
    rng = np.random.default_rng(200)
    first, second = rng.integers(0, 248320, 70).tolist(), rng.integers(0, 248320, 130).tolist()
    os.environ["Q38CU_TC_PREFILL"] = "0"
    try:
        dev.reset()
        dev.prefill(first)
        integer = dev.prefill(second)
    finally:
        del os.environ["Q38CU_TC_PREFILL"]
    dev.reset()
    dev.prefill(first)
    tc = dev.prefill(second)
    assert dev.position == 200
    ref.reset()
    ref.prefill(first)
    want = ref.prefill(second)
    check_logits(tc, want, "continued tensor-core prefill", cos_min=0.9)
    e_tc, e_int = rel(tc, want), rel(integer, want)
    print(f"continued prefill relative error vs upstream: tensor cores {e_tc:.3e}, integer path {e_int:.3e}")
    assert e_tc <= 1.5 * e_int + 1e-3, (e_tc, e_int)


def test_greedy_matches_upstream_teacher_forced(models, portable):
    """Greedy decoding under teacher forcing: the device and the upstream's
    portable build both read the native build's own greedy sequence.  The
    device's logits may drift from the native ones no further than the
    portable build's do (50 % slack), and its argmax must agree on the first
    steps wherever the native margin is safe.  Later steps are not held to
    top-1: on these conditioned weights a one-ulp difference doubles at every
    residual branch, so after a few tokens the two builds' logits differ by
    ~10 % (the free-running greedy test below uses a model built to be
    stable)."""
    dev, ref = models
    for m in (dev, ref, portable):
        m.reset()
    token = 1234
    dev_err, port_err = [], []
    dev_agree = port_agree = 0
    steps = 12
    for step in range(steps):
        want = ref.forward_token(token)
        got, alt = dev.forward_token(token), portable.forward_token(token)
        check_logits(got, want, f"greedy step {step}", cos_min=0.9, top1=False)
        if step < 2 and safe_margin(want):
            assert int(np.argmax(got)) == int(np.argmax(want)), f"greedy step {step}"
        dev_err.append(rel(got, want))
        port_err.append(rel(alt, want))
        dev_agree += int(np.argmax(got)) == int(np.argmax(want))
        port_agree += int(np.argmax(alt)) == int(np.argmax(want))
        token = int(np.argmax(want))
    assert np.mean(dev_err) <= 1.5 * np.mean(port_err) + 1e-3, (dev_err, port_err)
    print(f"teacher-forced greedy: device top-1 agrees on {dev_agree}/{steps}, portable on {port_agree}/{steps}")


def top2_margin(logits):
    s = np.sort(np.asarray(logits, np.float64))
    return (s[-1] - s[-2]) / max(abs(s[-1]), 1e-30)


@pytest.fixture(scope="module")
def robust_models():
    """The "robust" seeded model (gguf.py: residual branches damped, a peaked
    LM head) with the native and the portable upstream builds."""
    import os
    if not O.reference_available() or not os.path.exists(O.REF_PORTABLE_LIB):
        pytest.skip("upstream reference libraries not built")
    from q38b200.model import Model
    path = gguf.cached_model_path(seed=3, mtp=False, dist="robust")
    dev = Model(path, 128)
    nat = O.ReferenceModel(path, 128)
    por = O.ReferenceModel(path, 128, lib_path=O.REF_PORTABLE_LIB)
    yield dev, nat, por
    dev.close()
    nat.close()
    por.close()


def free_run(model, prompt, steps):
    """Greedy tokens and the logits each was chosen from."""
    model.reset()
    logits = model.prefill(prompt)
    tokens, seen = [], []
    for _ in range(steps):
        seen.append(logits)
        tokens.append(int(np.argmax(logits)))
        logits = model.forward_token(tokens[-1])
    return tokens, seen


def common_prefix(a, b):
    return next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), min(len(a), len(b)))


def test_free_running_greedy_matches_upstream(robust_models):
    """Free-running greedy decoding, 32 tokens after an 8-token prompt: the
    device's own loop (argmax fed back on the device) against the native
    upstream build's own greedy loop.  Two correct builds of this model are
    not bit-identical (every projection input is re-quantized to int8, so a
    one-ulp difference can flip an int8 and grow through the layers; the
    upstream's native and portable builds differ by a few percent in the
    logits), so the bar is the upstream's own: the device must reproduce the
    native tokens up to the first step the upstream itself finds ambiguous -
    where the native top-2 logit gap between the native choice and the
    device's is within 3x the native/portable difference at those entries,
    or where the portable build already left the native sequence.  Margins
    and both prefixes are printed."""
    dev, nat, por = robust_models
    prompt = np.random.default_rng(31).integers(0, 248320, 8).tolist()
    steps = 32
    nat_tokens, nat_logits = free_run(nat, prompt, steps)
    por_tokens, por_logits = free_run(por, prompt, steps)
    dev.reset()
    first = int(np.argmax(dev.prefill(prompt)))
    dev_tokens = [first] + dev.generate_greedy(first, steps - 1)
    k_dev, k_por = common_prefix(dev_tokens, nat_tokens), common_prefix(por_tokens, nat_tokens)
    print("native top-2 margins:", " ".join(f"{top2_margin(l):.3f}" for l in nat_logits))
    print(f"free-running greedy: device = native for {k_dev} of {steps} tokens, portable = native for {k_por}")
    if k_dev < steps and k_dev < k_por:
        n, d = nat_tokens[k_dev], dev_tokens[k_dev]
        gap = float(nat_logits[k_dev][n] - nat_logits[k_dev][d])
        spread = float(np.max(np.abs(nat_logits[k_dev][[n, d]] - por_logits[k_dev][[n, d]])))
        assert gap <= 3.0 * spread + 1e-6, (f"step {k_dev}: device {d} vs native {n}, native gap {gap:.4g} "
                                           f"beyond 3x the native/portable spread {spread:.4g}")
    assert dev_tokens[:k_dev] == nat_tokens[:k_dev]


def test_benchmark_model_layers_match_upstream():
    """The model bench.py times (config-0 draws, Q4_K_M mix, seed 0): layer 0
    against the upstream model (exact input), and every 4th layer plus every
    attention layer teacher-forced through the CPU restatement with the
    upstream's Q8_K kernels, over two tokens.  The config-0 draws are not
    conditioned (activations reach 1e5), so a one-ulp float difference inside
    a layer can flip a few int8 values of a later Q8_K activation: the bar is
    the in-layer flip bar (1e-2) with cosine above 0.9999, and most
    (layer, token) outputs must match to rounding (1e-5)."""
    if not O.reference_available():
        pytest.skip("upstream reference library not built")
    import model_oracle as MO
    from q38b200.model import Model
    path = gguf.cached_model_path(seed=0, mtp=True, dist="config0")
    dev = Model(path, 64)
    ref = O.ReferenceModel(path, 64)
    try:
        for token in (777, 3):
            dev.reset()
            ref.reset()
            got, want = dev.forward_token_layers(token, 1), ref.forward_token_layers(token, 1)
            assert np.all(np.isfinite(got))
            assert rel(got, want) <= 1e-2 and cosine(got, want) >= 0.9999, (rel(got, want), cosine(got, want))
        lo = MO.LayerOracle(path, O.Reference())
        tokens = (4321, 17)
        errors, cosines = [], []
        for layer in sorted(set(range(0, 64, 4)) | set(range(3, 64, 4))):
            dev.reset()
            inputs = [dev.forward_token_layers(t, layer) for t in tokens]
            dev.reset()
            outputs = [dev.forward_token_layers(t, layer + 1) for t in tokens]
            sl = MO.StatefulLayer(lo, layer)
            for i, o in zip(inputs, outputs):
                want = sl.step(i)
                errors.append(rel(o, want))
                cosines.append(cosine(o, want))
        errors = np.array(errors)
        print(f"benchmark model, teacher-forced: worst {errors.max():.2e}, exact {np.mean(errors <= 1e-5):.2f}")
        assert errors.max() <= 1e-2 and min(cosines) >= 0.9999
        assert np.mean(errors <= 1e-5) >= 0.5
    finally:
        dev.close()
        ref.close()


def test_device_greedy_loop_is_the_argmax_loop(models):
    dev, _ = models
    dev.reset()
    token, want = 99, []
    for _ in range(10):
        token = int(np.argmax(dev.forward_token(token)))
        want.append(token)
    dev.reset()
    assert dev.generate_greedy(99, 10) == want
    assert dev.position == 10


def test_mtp_head_after_prefill_matches_upstream(models):
    """Prefill with MTP enabled runs the MTP catch-up over every prompt token
    (chunks of 8 and 3 here); the next draft's logits then depend on all of it."""
    dev, ref = models
    prompt = np.random.default_rng(9).integers(0, 248320, 11).tolist()
    for m in (dev, ref):
        m.reset()
        m.enable_mtp()
    check_logits(dev.prefill(prompt), ref.prefill(prompt), "prefill with MTP", cos_min=0.9)
    check_logits(dev.mtp_forward(prompt[-1]), ref.mtp_forward(prompt[-1]), "MTP draft after prefill", cos_min=0.9)


@pytest.mark.parametrize("drafts", [1, 3, 8, 10])
def test_speculative_greedy_preserves_greedy(models, drafts):
    """q38_model_speculative_greedy keeps the target's exact greedy sequence
    (qwen38_model.h:33-36): drafts, batch verification, rollback of the
    recurrent state to the consumed prefix (up to 8 drafts; replay of the
    prefix beyond) and MTP catch-up must not change a single token, and the
    logits returned are those of the last consumed token."""
    dev, _ = models
    dev.reset()
    plain = dev.generate_greedy(7, 12)
    dev.reset()
    dev.enable_mtp()
    token, seq = 7, []
    while len(seq) < 12:
        accepted, logits = dev.speculative_greedy(token, 0xFFFFFFFF, drafts)
        assert 1 <= len(accepted) <= drafts
        assert int(np.argmax(logits)) == accepted[-1]
        seq += accepted
        token = accepted[-1]
    assert seq[:12] == plain
    assert dev.position == len(seq)


def test_iq1m_model_first_layer_matches_upstream():
    """The IQ1_M-typed variant (gguf mix "IQ1_M": IQ1_M for every Q4_K matrix
    but the embedding, config-0 weight draws): layer 0, a DeltaNet block whose
    qkv, gate, out, ffn_gate and ffn_up are IQ1_M, sees the exact embedding
    row.  The config-0 draws are not conditioned (the layer's activations
    reach 1e5), so a one-ulp difference in a float sum inside the layer flips
    a few int8 values of the later Q8_K activations: the bar is the in-layer
    flip bar of the teacher-forced test (1e-2; observed 3e-4), with the cosine
    above 0.9999.  A wrong decoder would be off by order 1."""
    if not O.reference_available():
        pytest.skip("upstream reference library not built")
    from q38b200.model import Model
    path = gguf.cached_model_path(seed=2, mtp=False, dist="config0", mix="IQ1_M")
    dev = Model(path, 64)
    ref = O.ReferenceModel(path, 64)
    try:
        for token in (777, 3):
            dev.reset()
            ref.reset()
            got, want = dev.forward_token_layers(token, 1), ref.forward_token_layers(token, 1)
            assert np.all(np.isfinite(got))
            assert rel(got, want) <= 1e-2 and cosine(got, want) >= 0.9999
    finally:
        dev.close()
        ref.close()
