"""Import path mirror of KVCache-Factory's ``pyramidkv`` package for the CircuitKV hook."""
