"""Shared test helpers."""


def word_tokenizer(vocab: int):
    """A tokenizer whose every id is one whitespace-separated word ``<i>`` (no word is part of another)."""
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    tok = Tokenizer(models.WordLevel({f"<{i}>": i for i in range(vocab)}, unk_token="<0>"))
    tok.pre_tokenizer = pre_tokenizers.WhitespaceSplit()
    tok.decoder = decoders.WordPiece(prefix="##", cleanup=False)
    return PreTrainedTokenizerFast(tokenizer_object=tok, unk_token="<0>", eos_token="<1>")
