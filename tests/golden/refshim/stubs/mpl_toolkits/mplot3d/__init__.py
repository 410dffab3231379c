Axes3D=None
