"""Tree construction, acceptance and the generate loop."""
