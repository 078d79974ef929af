"""Tokenised data: the vagus-tokens-v1 store, the window loader, preparation."""
from .loader import TokenStore, WindowLoader  # noqa: F401
