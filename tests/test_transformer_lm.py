"""Reference-shaped TransformerLM training step on the CPU path."""

from underhfs import tensor
from underhfs.functional import cross_entropy
from underhfs.nn import GELU, TransformerLM
from underhfs.optim import SGD


def test_gelu_grad_shape():
    x = tensor([-1.0, 0.0, 1.0], requires_grad=True)
    GELU()(x).sum().backward()
    assert x.grad.shape == x.shape


def test_one_sgd_step_changes_versions():
    lm = TransformerLM(vocab_size=8, max_seq_len=4, features=4, hidden_features=8, layers=1)
    opt = SGD(lm.parameters(), lr=1e-3)
    logits = lm(tensor([1, 2, 3, 4]))
    assert logits.shape == (4, 8)
    cross_entropy(logits, tensor([2, 3, 4, 5])).backward()
    assert any(p.grad is not None for p in lm.parameters())
    before = [p.version for p in lm.parameters()]
    opt.step()
    assert any(b > a for a, b in zip(before, [p.version for p in lm.parameters()]))


def test_loss_decreases_on_repeated_batch():
    from underhfs.optim import AdamW

    lm = TransformerLM(vocab_size=16, max_seq_len=8, features=8, hidden_features=16, layers=1, heads=2)
    opt = AdamW(lm.parameters(), lr=1e-2, weight_decay=0.0)
    ids, tg = tensor([[1, 2, 3, 4, 5, 6, 7, 8]]), tensor([[2, 3, 4, 5, 6, 7, 8, 9]])
    losses = []
    for _ in range(20):
        opt.zero_grad()
        loss = lm(ids, tg)
        losses.append(loss.item())
        loss.backward()
        opt.step()
    assert losses[-1] < losses[0] * 0.5
