class Module:
    def __init__(self):
        pass
