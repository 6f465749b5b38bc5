__version__ = "0.1.10+b200"
