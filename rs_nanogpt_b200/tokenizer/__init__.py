from .bpe import (SPECIAL_TOKENS, BpeTokenizer, TokenDecoder, Role, Part, Message, Conversation,  # noqa: F401
                  RenderedConversation)
