"""Interactive chat on top of A10Decoder (the reference's a10_chat.py:222-604).

Behaviour kept from the reference:
  * the ChatML prompt with the reference's system line (a10_chat.py:580-588):
    every turn re-sends the whole conversation, ending with an open assistant
    turn;
  * prompts longer than max_seq_len - max_new_tokens keep their last tokens
    (a10_chat.py:344-348);
  * greedy decoding until EOS or max_new_tokens; streamed output prints each
    token as it is decoded and ends with a prefill / decode speed line
    (a10_chat.py:444-549);
  * the reply is cut at <|im_end|> and <think>...</think> blocks are removed
    (a10_chat.py:593-599);
  * the REPL understands "quit" / "exit" and "clear" (a10_chat.py:551-604).
Differences: the prompt is prefilled 64 tokens per launch (INT8 decoder) instead
of one token per launch, and the I/O functions are parameters, so the loop can
be driven by tests or another front end.
"""
import re
import time

SYSTEM_LINE = "You are a helpful assistant. Be concise and direct. /nothink"


def format_prompt(conversation, system=SYSTEM_LINE):
    """ChatML prompt of a conversation [{"role": "user"|"assistant", "content": str}, ...]."""
    parts = [f"<|im_start|>system\n{system}<|im_end|>\n"]
    for msg in conversation:
        role = "user" if msg["role"] == "user" else "assistant"
        parts.append(f"<|im_start|>{role}\n{msg['content']}<|im_end|>\n")
    parts.append("<|im_start|>assistant\n")
    return "".join(parts)


def clean_response(text):
    """Reply text without the end-of-turn marker and without thinking blocks."""
    text = text.split("<|im_end|>")[0].strip()
    text = re.sub(r"<think>.*?</think>", "", text, flags=re.DOTALL).strip()
    if "<think>" in text:
        text = text.split("<think>")[0].strip()
    return text or "[Model is thinking... try asking more directly]"


class A10Chat:
    """Chat front end.  `decoder` is an A10Decoder built with a tokenizer (an
    object with encode(str) -> ids, decode(ids, skip_special_tokens=...) -> str
    and eos_token_id)."""

    def __init__(self, decoder, tokenizer=None):
        self.decoder = decoder
        self.tokenizer = tokenizer if tokenizer is not None else decoder.tokenizer
        if self.tokenizer is None:
            raise ValueError("A10Chat needs a tokenizer")
        self.conversation = []
        self.last_stats = None

    def _ids(self, prompt, max_new_tokens):
        if max_new_tokens <= 0:
            raise ValueError("max_new_tokens must be positive")
        ids = list(self.tokenizer.encode(prompt))
        limit = self.decoder.max_seq_len - max_new_tokens - 1
        if len(ids) > limit:
            ids = ids[-limit:]
        if not ids:
            raise ValueError("empty prompt")
        return ids

    def _decode_text(self, ids):
        return self.tokenizer.decode(ids, skip_special_tokens=True)

    def generate_stream(self, prompt, max_new_tokens=500, out=None):
        """Yields the text of each generated token; `out` (e.g. print) also gets it.
        Sets self.last_stats = (prompt_tokens, prefill_s, new_tokens, decode_s)."""
        ids = self._ids(prompt, max_new_tokens)
        eos = getattr(self.tokenizer, "eos_token_id", None)
        dec = self.decoder.decoder
        self.decoder.reset()
        t0 = time.perf_counter()
        if hasattr(dec, "prefill"):
            tok = dec.prefill(ids)
        else:
            tok = None
            for t in ids:
                tok = dec.decode_step(t)
        t1 = time.perf_counter()
        n = 0
        while True:
            n += 1
            piece = self._decode_text([tok])
            if out is not None:
                out(piece)
            yield piece
            if tok == eos or n >= max_new_tokens or dec.position() >= self.decoder.max_seq_len:
                break
            tok = dec.decode_step(tok)
        self.last_stats = (len(ids), t1 - t0, n, time.perf_counter() - t1)

    def generate(self, prompt, max_new_tokens=100, show_speed=True, out=print):
        """Whole reply (the reference's generate); prints the speed line when asked."""
        text = "".join(self.generate_stream(prompt, max_new_tokens))
        if show_speed and out is not None:
            out(self.speed_line())
        return text

    def speed_line(self):
        p, tp, n, td = self.last_stats
        return (f"[prefill: {p} tok @ {p / tp if tp > 0 else 0:.0f} tok/s | "
                f"decode: {n} tok @ {n / td if td > 0 else 0:.0f} tok/s | total: {(tp + td) * 1000:.0f}ms]")

    def turn(self, user_text, max_new_tokens=500, out=None):
        """One conversation turn: appends the user message, streams the reply,
        stores the cleaned reply in the history and returns it."""
        self.conversation.append({"role": "user", "content": user_text})
        raw = "".join(self.generate_stream(format_prompt(self.conversation), max_new_tokens, out=out))
        reply = clean_response(raw)
        self.conversation.append({"role": "assistant", "content": reply})
        return reply

    def chat(self, input_fn=input, print_fn=print, max_new_tokens=500):
        """The REPL: 'quit' / 'exit' ends it, 'clear' starts a new conversation."""
        print_fn("Qwen3-0.6B chat (B200 decode kernel). 'quit' or 'exit' ends, 'clear' starts over.")
        while True:
            try:
                user = input_fn("You: ").strip()
            except (KeyboardInterrupt, EOFError):
                print_fn("Goodbye!")
                return
            if not user:
                continue
            if user.lower() in ("quit", "exit"):
                print_fn("Goodbye!")
                return
            if user.lower() == "clear":
                self.conversation = []
                print_fn("[Conversation cleared]")
                continue
            reply = self.turn(user, max_new_tokens)
            print_fn("Assistant: " + reply)
            print_fn(self.speed_line())
