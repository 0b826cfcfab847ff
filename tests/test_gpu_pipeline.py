"""The long-audio pipeline (madi_b200/pipeline.py: conv stem, encoder layers,
ln_post, cross K / V, greedy decoder with EOT suppressed) on a reduced depth:
its size-independent properties, since every piece it chains is parity-tested
on its own (encoder layer, decoder end to end, attention, decode-step helpers):

* batch invariance -- a chunk's encoder states and tokens are the same whether
  it is processed in a batch of 4, of 2 or alone (per-row GEMM accumulation does
  not depend on M; attention and the decode kernels are per chunk / slot);
* determinism -- the same input gives the same tokens again;
* the forced length -- exactly `tokens` tokens, none of them EOT or a special.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tr(madi):
    from madi_b200 import pipeline
    t = pipeline.Transcriber(slots=4, enc_layers=2, tokens=6, seed=3)
    yield t
    t.release()


def test_stem_and_layer_batch_invariance(madi):
    """The stem (one convolution call per chunk) and one encoder layer (Q8 GEMMs
    at M = 4 x 1500 vs 1500, flash attention, LNs) each give a chunk the same
    bits in any batch."""
    import torch
    from madi_b200 import encoder as enc, pipeline
    e = enc.Encoder(layers=1, seed=5)
    mel = torch.from_numpy(pipeline.synthetic_mel(3, first=70)).cuda()
    x3 = torch.cat([e.stem(mel[i:i + 1]) for i in range(3)]).reshape(-1, enc.D).contiguous()
    x1 = e.stem(mel[1:2]).reshape(-1, enc.D).contiguous()
    assert torch.equal(x3[enc.SEQ:2 * enc.SEQ], x1)
    L = e.layers[0]
    f3 = L.forward(x3.clone(), None, None)
    f1 = L.forward(x1.clone(), None, None)
    torch.cuda.synchronize()
    assert torch.equal(f3[enc.SEQ:2 * enc.SEQ], f1), "encoder layer output depends on the batch"


def test_batch_invariance(tr):
    import torch
    from madi_b200 import pipeline
    mel = torch.from_numpy(pipeline.synthetic_mel(5, first=10)).cuda()
    states4 = tr.encode(mel[:4])
    states1 = torch.cat([tr.encode(mel[i:i + 1]) for i in range(4)])
    states2 = torch.cat([tr.encode(mel[0:2]), tr.encode(mel[2:4])])
    assert torch.equal(states4, states1) and torch.equal(states4, states2), "encoder states depend on the batch"
    tok_batch = torch.cat([tr.decode(states4).clone(), tr.transcribe(mel[4:5]).clone()])
    tok_single = torch.cat([tr.transcribe(mel[i:i + 1]).clone() for i in range(5)])
    torch.cuda.synchronize()
    assert torch.equal(tok_batch, tok_single), f"{tok_batch.tolist()} vs {tok_single.tolist()}"
    again = tr.transcribe(mel[:4]).clone()
    assert torch.equal(again, tok_batch[:4])


def test_forced_length(tr):
    import torch
    from madi_b200 import pipeline
    mel = torch.from_numpy(pipeline.synthetic_mel(3, first=40)).cuda()
    toks = tr.transcribe(mel).clone().cpu().numpy().view(np.uint32)
    assert toks.shape == (3, 6)
    assert (toks < pipeline.EOT).all(), toks
    assert int(tr.decoder.pos[0].item()) == 6


@pytest.mark.parametrize("act16", [False, True])
def test_slot_count_invariance(madi, act16):
    """The decoder at 12 slots (two token groups per GEMV weight fragment) gives the
    first 4 chunks the same tokens as the decoder at 4 slots (f32 or f16 activations)."""
    import torch
    from madi_b200 import decoder as dec
    w = dec.device_weights(seed=9)
    g = torch.Generator(device="cuda")
    g.manual_seed(17)
    states = torch.randn((12, dec.ENC, dec.D), device="cuda", generator=g).half()
    got = []
    for slots in (12, 4):
        d = dec.Decoder(w, slots, act16=act16)
        d.set_encoder(states[:slots].contiguous())
        d.reset(50258)
        for _ in range(6):
            d.step()
        torch.cuda.synchronize()
        got.append(d.tokens[:4, :7].clone())
        del d
    assert torch.equal(got[0], got[1]), f"{got[0].tolist()} vs {got[1].tolist()}"


def test_transcribe_chunks_overlap(tr):
    """transcribe_chunks (host mel in, host tokens out, batch k+1's encoder beside batch
    k's decoder) gives the tokens transcribe() gives batch by batch, overlapped or not."""
    import torch
    from madi_b200 import pipeline
    mel = pipeline.synthetic_mel(6, first=90)
    mel_h = torch.from_numpy(mel).pin_memory()
    got = []
    for overlap in (True, False):
        tok_h = torch.full((6, 6), -1, dtype=torch.int32).pin_memory()
        tr.transcribe_chunks(mel_h, tok_h, overlap=overlap)
        torch.cuda.synchronize()
        got.append(tok_h.clone())
    m = torch.from_numpy(mel).cuda()
    want = torch.cat([tr.transcribe(m[0:4]).cpu(), tr.transcribe(m[4:6]).cpu()])
    assert torch.equal(got[0], want) and torch.equal(got[1], want), f"{got[0].tolist()} vs {want.tolist()}"


def test_eight_step_graph_equals_eager_steps(madi):
    """With tokens a multiple of 8 the token step is captured eight times in one graph
    (the reference's DBATCH); replaying it gives the tokens of 16 eager steps."""
    import torch
    from madi_b200 import pipeline
    t = pipeline.Transcriber(slots=2, enc_layers=1, tokens=16, seed=4, decoders=1)
    assert t.steps_per_graph == 8
    mel = torch.from_numpy(pipeline.synthetic_mel(2, first=30)).cuda()
    states = t.encode(mel)
    got = t.decode(states).clone()
    d = t.decoders[0]
    d.reset(pipeline.SOT)
    for _ in range(16):
        d.step(suppress=t.eot)
    torch.cuda.synchronize()
    assert torch.equal(got, d.tokens[:2, 1:17])
    assert int(d.pos[0].item()) == 16
    t.release()
