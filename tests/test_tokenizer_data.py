"""Tokenizers and file-backed data."""
import torch

from burn_dragon_b200.train.data import FileBytes, RandomBytes, StreamingBytes
from burn_dragon_b200.utils.tokenizer import BPETokenizer, ByteTokenizer, load_tokenizer


def test_byte_tokenizer_round_trip():
    t = ByteTokenizer()
    s = "héllo, dragon 🐉"
    assert t.decode(t.encode(s)) == s


def test_bpe_train_encode_decode():
    corpus = ["the dragon hatchling hatches the dragon egg"] * 20 + ["low lower lowest"] * 10
    tok = BPETokenizer().train(corpus, 300)
    assert 256 < tok.vocab_size <= 300
    s = "the dragon hatchling is lowest"
    ids = tok.encode(s)
    assert tok.decode(ids) == s
    assert len(ids) < len(s.encode())  # merges compress frequent words
    again = load_tokenizer(tok.to_json())
    assert again.encode(s) == ids


def test_random_and_streaming_loaders_are_seeded():
    a = RandomBytes(2, 8, seed=3, rank=0, world=2).next()
    b = RandomBytes(2, 8, seed=3, rank=1, world=2).next()
    assert not torch.equal(a[0], b[0])
    assert torch.equal(a[0], RandomBytes(2, 8, seed=3, rank=0, world=2).next()[0])
    s = StreamingBytes(3, 64, 16, seed=1)
    x1, y1, r1 = s.next()
    x2, _, r2 = s.next()
    assert r1 and not r2 and torch.equal(y1[:, -1], x2[:, 0])


def test_file_bytes(tmp_path):
    p = tmp_path / "corpus.bin"
    p.write_bytes(bytes(range(256)) * 20)
    tr = FileBytes(str(p), 4, 16)
    x, y = tr.next()
    assert x.shape == (4, 16) and torch.equal((x[:, 1:]), y[:, :-1])
    va = FileBytes(str(p), 2, 16, split="valid")
    assert va.next()[0].shape == (2, 16)
