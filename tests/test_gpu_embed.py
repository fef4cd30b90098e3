"""The real tokens' embedding in one launch (tb_embed_rows) against PyTorch's index_select +
embedding + cast (reference: solution/model.py:220-225), bit for bit; a token id outside the
vocabulary, which the kernel's bounds check turns into a zero row and a counted error."""

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("batch,seq,hidden,vocab", [(4, 512, 1536, 151936), (3, 40, 256, 1000),
                                                    (1, 1, 8, 17)])
def test_embedding_matches_torch(batch, seq, hidden, vocab):
    from testt_b200.model import embed_rows

    g = torch.Generator().manual_seed(hidden)
    ids = torch.randint(0, vocab, (batch, seq), generator=g).to(DEV)
    table = (torch.randn(vocab, hidden, generator=g) * 0.02).half().to(DEV)
    n = max(1, batch * seq * 2 // 3)
    pos = torch.randperm(batch * seq, generator=g)[:n].sort().values.to(DEV)
    got = embed_rows(ids, pos, table)
    ref = torch.nn.functional.embedding(ids.reshape(-1).index_select(0, pos), table).float()
    torch.cuda.synchronize()
    assert got.dtype == torch.float32
    assert torch.equal(got, ref)


def test_out_of_range_id_gives_a_zero_row_and_is_counted():
    from testt_b200 import _lib

    lib = _lib.load()
    table = torch.randn(10, 16, device=DEV).half()
    ids = torch.tensor([3, 12, -1, 9], dtype=torch.int64, device=DEV)
    pos = torch.arange(4, device=DEV)
    out = torch.full((4, 16), 5.0, device=DEV)
    before = lib.tb_embed_invalid_ids()
    _lib.call("tb_embed_rows", _lib.ptr(ids), _lib.ptr(pos), _lib.ptr(table), _lib.ptr(out), 4,
              16, 10, _lib.stream_of(out))
    torch.cuda.synchronize()
    assert lib.tb_embed_invalid_ids() == before + 2
    assert torch.equal(out[0], table[3].float()) and torch.equal(out[3], table[9].float())
    assert torch.all(out[1:3] == 0)
