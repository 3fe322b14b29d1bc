"""Kernel-level parity on the B200: tcgen05 GEMM, tcgen05 attention, STFT / iSTFT.

Each kernel runs through the C-ABI stage entry points and is compared with a
float32/float64 reference of the same op on the same (16-bit-representable)
inputs.  Tolerances are stated per test.
"""

import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from karaoke_platform_sidecar_native_b200 import native  # noqa: E402
from oracle import vocalarc_oracle as O  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def provider():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    p = native.Provider(0)
    yield p
    p.close()


def run(provider, fn, *args):
    torch.cuda.synchronize()
    fn(*args)
    provider.synchronize()
    assert provider.take_device_error() == 0


def rel_max(a, b):
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


@pytest.mark.parametrize("m,n,k", [(1, 256, 64), (127, 256, 256), (128, 256, 256), (129, 1536, 256),
                                   (1000, 256, 512), (4097, 1024, 256), (777, 256, 1024)])
def test_gemm_fp32_out(provider, m, n, k):
    # C = A B^T with fp16 operands; reference: fp32 product of the same fp16 values.
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n)
    a = torch.randn(m, k, device="cuda", generator=g).half()
    b = (torch.randn(n, k, device="cuda", generator=g) * 0.05).half()
    out = torch.full((m, n), float("nan"), device="cuda")
    run(provider, provider.stage_gemm, 6, a, b, m, n, k, None, out)
    ref = a.float() @ b.float().T
    assert rel_max(out, ref) < 1e-5   # fp32 accumulation order only


@pytest.mark.parametrize("epilogue", [0, 1])
def test_gemm_f16_bias_and_gelu(provider, epilogue):
    m, n, k = 1537, 1024, 256
    g = torch.Generator(device="cuda").manual_seed(11 + epilogue)
    a = torch.randn(m, k, device="cuda", generator=g).half()
    b = (torch.randn(n, k, device="cuda", generator=g) * 0.05).half()
    bias = torch.randn(n, device="cuda", generator=g) * 0.1
    out = torch.zeros(m, n, device="cuda", dtype=torch.float16)
    run(provider, provider.stage_gemm, epilogue, a, b, m, n, k, bias, out)
    ref = a.float() @ b.float().T + bias
    if epilogue == 1:
        ref = torch.nn.functional.gelu(ref)   # exact erf GELU
    assert rel_max(out.float(), ref) < 2e-3   # fp16 output rounding (2^-11)


def attention_reference(qkv, gates, d1, d2, d3, pos_dim):
    x = qkv.float().view(d3, d2, d1, 1536)
    if pos_dim == 1:
        seqs = x.reshape(d3 * d2, d1, 1536)
    else:
        seqs = x.permute(0, 2, 1, 3).reshape(d3 * d1, d2, 1536)
    s, length = seqs.shape[0], seqs.shape[1]
    q = seqs[..., :512].reshape(s, length, 8, 64).transpose(1, 2)
    k = seqs[..., 512:1024].reshape(s, length, 8, 64).transpose(1, 2)
    v = seqs[..., 1024:].reshape(s, length, 8, 64).transpose(1, 2)
    att = torch.softmax((q @ k.transpose(-1, -2)) * 0.125, dim=-1) @ v     # [s][8][L][64]
    att = att.transpose(1, 2)                                                # [s][L][8][64]
    if pos_dim == 1:
        att = att.reshape(d3, d2, d1, 8, 64)
    else:
        att = att.reshape(d3, d1, d2, 8, 64).permute(0, 2, 1, 3, 4)
    att = att.reshape(-1, 8, 64) * gates.view(-1, 8, 1)
    return att.reshape(-1, 512)


@pytest.mark.parametrize("d1,d2,d3,pos_dim", [
    (1, 3, 1, 1), (2, 5, 2, 1), (87, 4, 1, 1), (128, 2, 1, 1), (129, 3, 1, 1), (300, 2, 2, 1), (862, 2, 1, 1),
    (1722, 3, 1, 1), (1723, 2, 1, 1),     # the benchmark's chunk length (14 key tiles, 58-row tail) and one more
    (7, 90, 1, 2), (26, 90, 2, 2), (3, 62, 1, 2), (5, 1, 1, 2), (9, 2, 1, 2)])
def test_attention_matches_fp32_softmax(provider, d1, d2, d3, pos_dim):
    rows = d1 * d2 * d3
    g = torch.Generator(device="cuda").manual_seed(rows + pos_dim)
    qkv = torch.randn(rows, 1536, device="cuda", generator=g).half()
    gates = torch.rand(rows, 8, device="cuda", generator=g)
    out = torch.full((rows, 512), float("nan"), device="cuda", dtype=torch.float16)
    run(provider, provider.stage_attention, qkv, gates, out, d1, d2, d3, pos_dim)
    ref = attention_reference(qkv, gates, d1, d2, d3, pos_dim)
    assert torch.isfinite(out.float()).all()
    # P is rounded to fp16 before P.V (relative 2^-11 per weight) and the output to fp16.
    assert rel_max(out.float(), ref) < 1e-2
    assert float((out.float() - ref).abs().mean() / ref.abs().mean()) < 2e-3


@pytest.mark.parametrize("d1,d2", [(1722, 2), (300, 3)])
def test_attention_rising_scores(provider, d1, d2):
    # Keys grow along the sequence (x1 to x7), so later key tiles score far
    # above a row's first tile: the time-axis kernel must raise its reference
    # maximum again and again, rescaling O in tensor memory and the packed P of
    # the tile's first half.
    rows = d1 * d2
    g = torch.Generator(device="cuda").manual_seed(7 + d1)
    qkv = torch.randn(rows, 1536, device="cuda", generator=g)
    ramp = 1.0 + 6.0 * torch.arange(d1, device="cuda", dtype=torch.float32) / d1
    qkv[:, 512:1024] *= ramp.repeat(d2)[:, None]
    qkv = qkv.half()
    gates = torch.rand(rows, 8, device="cuda", generator=g)
    out = torch.full((rows, 512), float("nan"), device="cuda", dtype=torch.float16)
    run(provider, provider.stage_attention, qkv, gates, out, d1, d2, 1, 1)
    ref = attention_reference(qkv, gates, d1, d2, 1, 1)
    assert torch.isfinite(out.float()).all()
    assert rel_max(out.float(), ref) < 1e-2
    assert float((out.float() - ref).abs().mean() / ref.abs().mean()) < 2e-3


def snr_db(ref, test):
    ref = np.asarray(ref, dtype=np.float64)
    err = ref - np.asarray(test, dtype=np.float64)
    return 10 * math.log10((ref ** 2).sum() / max((err ** 2).sum(), 1e-300))


@pytest.mark.parametrize("length", [300, 1000, 13230, 44100])
def test_stft_matches_oracle(provider, length):
    rng = np.random.default_rng(length)
    audio = (rng.standard_normal((2, 2, length)) * 0.1).astype(np.float32)      # two segments
    frames = length // 512 + 1
    d_audio = torch.from_numpy(audio).cuda()
    d_spec = torch.zeros(2, frames, 1025, 2, 2, device="cuda")
    run(provider, provider.stage_stft, d_audio, 2, length, d_spec)
    spec = d_spec.cpu().numpy()
    for seg in range(2):
        ref = O.stft(audio[seg])                                              # [1025][2][T][2]
        ours = spec[seg].transpose(1, 2, 0, 3)                                # -> [1025][2][T][2]
        assert snr_db(ref, ours) > 110   # fp32 FFT vs the reference's float64 FFT


@pytest.mark.parametrize("length", [300, 13230, 44100])
def test_istft_matches_oracle(provider, length):
    rng = np.random.default_rng(length + 1)
    audio = (rng.standard_normal((2, length)) * 0.1).astype(np.float32)
    source = O.stft(audio)
    mask = (rng.standard_normal(source.shape) * 0.3).astype(np.float32)
    ref = O.istft(source, mask, length)
    to_fm = lambda a: np.ascontiguousarray(a.transpose(2, 0, 1, 3))[None]     # [1][T][1025][2][2]
    d_spec = torch.from_numpy(to_fm(source)).cuda()
    d_mask = torch.from_numpy(to_fm(mask)).cuda()
    d_out = torch.zeros(1, 2, length, device="cuda")
    run(provider, provider.stage_istft, d_spec, d_mask, 1, length, d_out)
    assert snr_db(ref, d_out.cpu().numpy()[0]) > 100


@pytest.fixture(scope="module")
def provider_bf16():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    p = native.Provider(0)
    p.set_precision(True)
    yield p
    p.close()


@pytest.mark.parametrize("pos_dim", [1, 2])
def test_attention_config4_shapes_bf16(provider_bf16, pos_dim):
    # Config 4 op-level shapes, bf16 N(0,1) inputs: time axis 992 sequences x 801
    # tokens (62 bands x 16 chunks), band axis 12816 sequences x 62 tokens.  The
    # whole launch runs; 24 sequences are checked against an fp32 softmax of
    # the same bf16 values (P is rounded to bf16 before P.V: 2^-8 relative).
    d1, d2, d3 = 801, 62, 16
    rows = d1 * d2 * d3
    g = torch.Generator(device="cuda").manual_seed(4 + pos_dim)
    qkv = torch.randn(rows, 1536, device="cuda", generator=g).bfloat16()
    gates = torch.rand(rows, 8, device="cuda", generator=g)
    out = torch.full((rows, 512), float("nan"), device="cuda", dtype=torch.bfloat16)
    run(provider_bf16, provider_bf16.stage_attention, qkv, gates, out, d1, d2, d3, pos_dim)
    assert torch.isfinite(out.float()).all()
    x = qkv.view(d3, d2, d1, 1536)
    o = out.view(d3, d2, d1, 512)
    gt = gates.view(d3, d2, d1, 8)
    idx = torch.Generator().manual_seed(9)
    for _ in range(24):
        c = int(torch.randint(d3, (1,), generator=idx))
        if pos_dim == 1:
            b = int(torch.randint(d2, (1,), generator=idx))
            sel = (c, b, slice(None))
        else:
            f = int(torch.randint(d1, (1,), generator=idx))
            sel = (c, slice(None), f)
        ref = attention_reference(x[sel].contiguous(), gt[sel].contiguous(), x[sel].shape[0], 1, 1, 1)
        got = o[sel].float()
        assert rel_max(got, ref) < 3e-2
        assert float((got - ref).abs().mean() / ref.abs().mean()) < 8e-3
