"""Device LM-head argmax without allocation vs the host argmax entry point.

llmx_lm_head_argmax_device (device scratch in a fixed array, nothing allocated
per call) must return the same tokens as llmx_model_lm_head_argmax (the
restatement of model_data_t::lm_head_argmax, host/host_qwen_8x64.cpp:937-977):
exact int64 scores, first maximum wins, so the tolerance is zero.  Two calls in
a row share the scratch array.  Collected last so it also runs after every
other test in one process.
"""

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_lm_head_argmax_device_matches_host(llmx):
    torch = pytest.importorskip("torch")
    s = llmx.shape("qwen2.5-3b", layers=1)
    m = llmx.Model(s).init_gaussian(20260718, 0.02)  # tied N(0,1) Q8.8 embedding as LM head
    rng = np.random.default_rng(11)
    h1 = np.clip(rng.normal(0, 700, (1, s.hidden)), -32768, 32767).astype(np.int16)
    h8 = np.clip(rng.normal(0, 700, (8, s.hidden)), -32768, 32767).astype(np.int16)
    h8[3] = 0                 # every score 0: the first token must win
    h8[5] = h8[0]             # duplicate row
    h8[6, :] = 32767          # saturated row
    want1 = [m.lm_head_argmax(r) for r in h1]  # materialises the tied table
    want8 = [m.lm_head_argmax(r) for r in h8]
    p = llmx.lib().llmx_model_embedding(m.h)
    assert p, "tied embedding table not resident"
    table = np.ctypeslib.as_array(p, shape=(s.vocab, s.hidden))

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    w = torch.from_numpy(table.copy()).to(dev)
    d1 = torch.from_numpy(h1).to(dev)
    d8 = torch.from_numpy(h8).to(dev)
    t1 = torch.zeros(1, dtype=torch.int32, device=dev)
    t8 = torch.zeros(8, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    torch.cuda.synchronize()

    rc = llmx.lm_head_argmax_device(d1.data_ptr(), 1, s.hidden, w.data_ptr(), s.vocab, t1.data_ptr(), stream)
    assert rc == llmx.OK, llmx.last_error()
    rc = llmx.lm_head_argmax_device(d8.data_ptr(), 8, s.hidden, w.data_ptr(), s.vocab, t8.data_ptr(), stream)
    assert rc == llmx.OK, llmx.last_error()
    torch.cuda.synchronize()
    assert t1.cpu().numpy().astype(np.uint32).tolist() == want1
    assert t8.cpu().numpy().astype(np.uint32).tolist() == want8
    assert want8[3] == 0

    # the one- / two-vocabulary-row-per-warp variants (rows 2 and 3 -> 4) on
    # row subsets; after the first call's set-up no call allocates device memory
    for n in (2, 3):
        tn = torch.zeros(n, dtype=torch.int32, device=dev)
        torch.cuda.synchronize()
        free1 = torch.cuda.mem_get_info(dev)[0]
        rc = llmx.lm_head_argmax_device(d8.data_ptr(), n, s.hidden, w.data_ptr(), s.vocab, tn.data_ptr(), stream)
        assert rc == llmx.OK, llmx.last_error()
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info(dev)[0] == free1, "the call allocated device memory"
        assert tn.cpu().numpy().astype(np.uint32).tolist() == want8[:n]

    # more rows than the scratch holds: rejected before any launch
    rc = llmx.lm_head_argmax_device(d8.data_ptr(), 9, s.hidden, w.data_ptr(), s.vocab, t8.data_ptr(), stream)
    assert rc == llmx.ERR_ARG and "rows must be 1..8" in llmx.last_error()
