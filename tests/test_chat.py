"""Chat front end (megaqwen_b200/chat.py, the reference's a10_chat.py:222-604):
prompt format, reply cleaning, prompt truncation, stop at EOS, the REPL commands
(CPU, with a scripted decoder), and one turn on the GPU decoder."""
import pytest

from megaqwen_b200.chat import A10Chat, clean_response, format_prompt


class Tok:
    """Tokenizer stand-in: one id per character, id 0 = EOS."""
    eos_token_id = 0

    def encode(self, s):
        return [ord(ch) for ch in s]

    def decode(self, ids, skip_special_tokens=True):
        return "".join(chr(i) for i in ids if i != 0)


class ScriptedDecoder:
    """Mimics A10Decoder: replies with a fixed id sequence, then EOS."""

    def __init__(self, reply, max_seq_len=4096):
        self.max_seq_len, self.reply, self.tokenizer = max_seq_len, reply, Tok()
        self.decoder = self
        self.seen = []

    def reset(self):
        self.pos, self.k = 0, 0

    def prefill(self, ids):
        self.seen.append(list(ids))
        self.pos = len(ids)
        return self._next()

    def _next(self):
        self.k += 1
        return self.reply[self.k - 1] if self.k <= len(self.reply) else 0

    def decode_step(self, tok):
        self.pos += 1
        return self._next()

    def position(self):
        return self.pos


def test_format_prompt_is_chatml():
    p = format_prompt([{"role": "user", "content": "hi"}, {"role": "assistant", "content": "yo"}])
    assert p.startswith("<|im_start|>system\n") and p.endswith("<|im_start|>assistant\n")
    assert "<|im_start|>user\nhi<|im_end|>\n<|im_start|>assistant\nyo<|im_end|>\n" in p


def test_clean_response():
    assert clean_response("<think>x\ny</think> Hello<|im_end|>junk") == "Hello"
    assert clean_response("answer <think>unfinished") == "answer"
    assert clean_response("<think>only</think>").startswith("[Model is thinking")


def test_turns_keep_history_and_stop_at_eos():
    d = ScriptedDecoder([ord(c) for c in "Hi!"])
    chat = A10Chat(d)
    got = []
    assert chat.turn("hello", out=got.append) == "Hi!"
    assert "".join(got) == "Hi!" and chat.last_stats[2] == 4        # 3 characters + EOS
    chat.turn("again")
    assert [m["role"] for m in chat.conversation] == ["user", "assistant", "user", "assistant"]
    assert "Hi!" in Tok().decode(d.seen[-1])                        # the second prompt carries the history


def test_long_prompt_keeps_its_tail():
    d = ScriptedDecoder([ord("a")], max_seq_len=64)
    chat = A10Chat(d)
    "".join(chat.generate_stream("x" * 100 + "END", max_new_tokens=10))
    assert len(d.seen[-1]) == 64 - 10 - 1 and Tok().decode(d.seen[-1]).endswith("END")


def test_repl_commands():
    d = ScriptedDecoder([ord("o"), ord("k")])
    chat = A10Chat(d)
    script = iter(["", "hello", "clear", "hello", "quit"])
    lines = []
    chat.chat(input_fn=lambda _: next(script), print_fn=lines.append)
    assert "Assistant: ok" in lines and "[Conversation cleared]" in lines and lines[-1] == "Goodbye!"
    assert len(chat.conversation) == 2


@pytest.mark.gpu
def test_chat_turn_on_the_gpu_decoder():
    import megaqwen_b200 as mq

    class VocabTok(Tok):
        def encode(self, s):
            return [1000 + ord(ch) for ch in s]

        def decode(self, ids, skip_special_tokens=True):
            return "".join(chr(33 + i % 90) for i in ids)

    st = mq.make_synthetic_state(seed=3, num_layers=2)
    dec = mq.A10Decoder(st, quantized=True, max_seq_len=256, num_layers=2, tokenizer=VocabTok())
    chat = A10Chat(dec)
    reply = "".join(chat.generate_stream(format_prompt([{"role": "user", "content": "hi"}]), max_new_tokens=8))
    ids = VocabTok().encode(format_prompt([{"role": "user", "content": "hi"}]))
    want = dec.generate(ids, max_new_tokens=8)[len(ids):]   # decoded text, one character per id
    assert reply == want and len(reply) == 8
