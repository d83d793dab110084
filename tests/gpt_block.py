"""A nanoGPT-shaped language model of one block, written against a torch-like namespace, for the
drive-path tests: token and position embeddings, layer norms, causal self-attention through
``F.scaled_dot_product_attention`` on (B, H, L, D) head views, a GELU MLP and a head tied to
the token embedding, with a cross-entropy loss -- the ops DenseCore's tiny-GPT test trains
(tests/test_optim_exact.py:41-63 in the reference) and nanoGPT's model.py uses. ``T`` is the
module that plays ``torch`` and ``F`` the one that plays ``torch.nn.functional``."""


def make_gpt(T, F, vocab, n, heads, block):
    class GPT(T.nn.Module):
        def __init__(self):
            super().__init__()
            self.tok, self.pos = T.nn.Embedding(vocab, n), T.nn.Embedding(block, n)
            self.ln_attn, self.ln_mlp, self.ln_out = T.nn.LayerNorm(n), T.nn.LayerNorm(n), T.nn.LayerNorm(n)
            self.qkv, self.proj = T.nn.Linear(n, 3 * n, bias=False), T.nn.Linear(n, n, bias=False)
            self.up, self.down = T.nn.Linear(n, 4 * n), T.nn.Linear(4 * n, n)
            self.head = T.nn.Linear(n, vocab, bias=False)
            self.head.weight = self.tok.weight

        def forward(self, idx, targets):
            B, L = idx.shape
            x = self.tok(idx) + self.pos(T.arange(0, L, dtype=T.long, device=idx.device))
            q, k, v = self.qkv(self.ln_attn(x)).split(n, dim=2)
            q, k, v = (t.view(B, L, heads, n // heads).transpose(1, 2) for t in (q, k, v))
            y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
            x = x + self.proj(y.transpose(1, 2).contiguous().view(B, L, n))
            x = x + self.down(F.gelu(self.up(self.ln_mlp(x))))
            logits = self.head(self.ln_out(x))
            return F.cross_entropy(logits.view(-1, vocab), targets.view(-1), ignore_index=-1)

    return GPT()
