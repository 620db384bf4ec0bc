"""The GPU indexing process on a B200: it runs the route encoder's own CUDA
parameters (received as IPC handles, so no copy is made), gives the parent's
embeddings, sees an in-place weight change of the parent, and abandons a
chunk when the grant byte is cleared."""
import tempfile

import numpy as np
import pytest
import torch

from deltaserve_vllm_b200.adapters.routing.encoder import SentenceEncoder
from deltaserve_vllm_b200.adapters.routing.index_process import EncoderProcess, IndexGrant, Preempted

from test_indexing_process_cpu import TEXTS, tiny_bert_dir

pytestmark = pytest.mark.gpu


def test_gpu_process_shares_cuda_weights():
    with tempfile.TemporaryDirectory() as d:
        tiny_bert_dir(d)
        parent = SentenceEncoder(d, "query: ", 32, "cuda:0")
        want = parent.encode(TEXTS[:16])
        grant = IndexGrant()
        grant.set(True)
        before = torch.cuda.memory_allocated(0)
        ex = EncoderProcess(SentenceEncoder(d, "query: ", 32, "cuda:0"), "cuda:0",
                            shared=parent.shared_state(), grant=grant, low_priority=False, name="gpu").start()
        try:
            assert torch.cuda.memory_allocated(0) == before       # nothing copied in this process
            assert ex.info["layers_checked"] == 3
            np.testing.assert_allclose(ex.encode(TEXTS[:16]), want, rtol=0, atol=2e-2)
            with torch.no_grad():
                parent._model.embeddings.word_embeddings.weight.mul_(-1.0)
            torch.cuda.synchronize()
            np.testing.assert_allclose(ex.encode(TEXTS[:4]), parent.encode(TEXTS[:4]), rtol=0, atol=2e-2)
            grant.set(False)
            with pytest.raises(Preempted):
                ex.encode(TEXTS[:4])
        finally:
            ex.stop()
