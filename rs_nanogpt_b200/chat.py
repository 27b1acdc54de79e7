"""`chat`: a REPL over a finetuned checkpoint (rs-nanogpt src/chat.rs:71-235).

Commands: ``quit``/``exit`` leave, ``clear`` starts a new conversation, EOF
exits; ``--prompt`` answers one prompt and exits. Each turn appends
``<|user_start|> text <|user_end|> <|assistant_start|>`` to the history,
refuses when the context is full, warns when the reply must be cut short,
streams the reply through a UTF-8-safe decoder, drops a trailing BOS and
forces a closing ``<|assistant_end|>`` into the history.
"""
import sys

import torch

from .eval.sample import SampleOptions, cached_model, generate_ids
from .tokenizer import BpeTokenizer
from .utils import checkpoint


def chat_turn(model, tok: BpeTokenizer, opts_base: SampleOptions, ids, text: str, out) -> None:
    seq_len = model.cfg.sequence_len
    base = len(ids)
    tok.push_user_turn(ids, text)
    room = max(0, seq_len - len(ids))
    if room == 0:
        del ids[base:]
        out.write(f"\n[this turn does not fit the model's {seq_len}-token context; type 'clear' to start over]\n")
        return
    max_tokens = min(opts_base.max_tokens, room)
    if max_tokens < opts_base.max_tokens:
        out.write(f"\n[only {max_tokens} of the {seq_len}-token context are left; the reply will be cut short]\n")
    out.write("\nAssistant: ")
    out.flush()
    dec = tok.decode_stream()
    stop = tok.assistant_stop_ids()
    opts = SampleOptions(max_tokens, opts_base.temperature, opts_base.top_k, opts_base.seed)

    def on_token(t):
        out.write(dec.push(t))
        out.flush()

    gen = generate_ids(model, ids, opts, stop, on_token)
    out.write(dec.finish() + "\n")
    assistant_end, bos = stop
    if gen and gen[-1] == bos:
        gen.pop()
    if not gen or gen[-1] != assistant_end:
        gen.append(assistant_end)
    ids.extend(gen)


def repl(model, tok: BpeTokenizer, opts: SampleOptions, prompt, inp=sys.stdin, out=sys.stdout) -> None:
    ids = [tok.bos_id()]
    while True:
        if prompt is not None:
            text = prompt.strip()
        else:
            out.write("\nUser: ")
            out.flush()
            line = inp.readline()
            if line == "":
                out.write("\nGoodbye!\n")
                return
            text = line.strip()
        low = text.lower()
        if low in ("quit", "exit"):
            out.write("Goodbye!\n")
            return
        if low == "clear":
            ids = [tok.bos_id()]
            out.write("conversation cleared\n")
        elif text:
            chat_turn(model, tok, opts, ids, text, out)
        if prompt is not None:
            return


def run_chat(args) -> None:
    device = torch.device(args.device or ("cuda" if torch.cuda.is_available() else "cpu"))
    meta = checkpoint.load_meta(args.checkpoint)
    tok = BpeTokenizer.from_file(args.vocab)
    if tok.vocab_size() != meta.config.vocab_size:
        raise ValueError(f"vocabulary size mismatch: {args.vocab} defines {tok.vocab_size()} tokens, the "
                         f"checkpoint expects {meta.config.vocab_size}. Pass the vocab file the checkpoint was "
                         "trained with")
    store, _ = checkpoint.load(args.checkpoint, device)
    model = cached_model(store)
    print(f"chat: {args.checkpoint} | step {meta.step} | val_bpb {meta.val_bpb:.4f} | context "
          f"{meta.config.sequence_len} tokens")
    print(f"sampling: temperature {args.temperature} | top_k {args.top_k} | max_tokens {args.max_tokens} | "
          f"seed {args.seed}")
    print("commands: 'clear' starts a new conversation, 'quit' or Ctrl-D exits")
    repl(model, tok, SampleOptions(args.max_tokens, args.temperature, args.top_k, args.seed), args.prompt)
