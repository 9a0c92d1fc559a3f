"""Test infrastructure: a deterministic character-level stand-in for an HF tokenizer (the HF
tokenizers of the reference's checkpoints are not available offline). Each character maps to one
id; decoding writes the ids out. Shared by the server fixture generator and the server test."""


class StubTokenizer:
    def __init__(self, vocab):
        self.vocab = vocab

    class _Enc:
        def __init__(self, ids):
            self.input_ids = ids

    def __call__(self, text, add_special_tokens=False, split_special_tokens=False):
        return self._Enc([(ord(c) * 131 + 7) % self.vocab for c in text])

    def decode(self, ids):
        return " ".join(str(int(i)) for i in ids)


# The server fixture's requests: (prefix, documents, suffix, tenant, max_tokens, recompute_ratio, policy).
SERVER_REQUESTS = (
    ("You are a careful assistant. ", ["alpha doc about rivers and lakes", "beta doc on mountains",
                                       "gamma doc: deserts, dunes and oases"], "Q: which is driest? A:", "", 12,
     0.0, "deviation"),
    ("You are a careful assistant. ", ["gamma doc: deserts, dunes and oases", "alpha doc about rivers and lakes",
                                       "beta doc on mountains"], "Q: which is wettest? A:", "", 12, 0.2, "deviation"),
    ("You are a careful assistant. ", ["beta doc on mountains", "delta doc about glaciers in winter"],
     "Q: which is coldest? A:", "", 10, 0.5, "boundary"),
    ("You are a careful assistant. ", ["alpha doc about rivers and lakes", "beta doc on mountains"],
     "Q: rivers? A:", "tenant-b", 8, 0.2, "deviation"),
    ("You are a careful assistant. ", ["gamma doc: deserts, dunes and oases", "beta doc on mountains",
                                       "alpha doc about rivers and lakes"], "Q: which is driest? A:", "", 12, 0.2,
     "deviation"),
)
