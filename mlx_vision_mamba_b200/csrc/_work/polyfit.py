import numpy as np
deg=int(__import__('sys').argv[1]) if len(__import__('sys').argv)>1 else 6
a,b=-0.5,0.5
xs=np.cos(np.pi*(np.arange(4000)+0.5)/4000)*0.5
ys=np.exp2(xs)
# Lawson iterations for minimax relative error
w=np.ones_like(xs)
V=np.vander(xs,deg+1,increasing=True)
for it in range(200):
    W=np.sqrt(w)/ys
    c,*_=np.linalg.lstsq(V*W[:,None], ys*W, rcond=None)
    err=np.abs(V@c-ys)/ys
    w=w*err; w/=w.sum()
c32=c.astype(np.float32)
# evaluate fp32 Horner with fma emulation on a dense grid
grid=np.linspace(-0.5,0.5,2000001).astype(np.float32)
def horner(f):
    p=np.full_like(f,c32[deg])
    for k in range(deg-1,-1,-1):
        p=(p.astype(np.float64)*f.astype(np.float64)+np.float64(c32[k])).astype(np.float32)
    return p
p=horner(grid)
ex=np.exp2(grid.astype(np.float64))
rel=(p.astype(np.float64)-ex)/ex
ulp=np.abs(np.spacing(ex.astype(np.float32))).astype(np.float64)
e_ulp=(p.astype(np.float64)-ex)/ulp
print('deg',deg,'coeffs',[float(x) for x in c32])
print('max rel (fp64 poly)',np.max(np.abs(V@c-ys)/ys))
print('fp32 Horner: max |err| ulp %.3f mean err ulp %.4f'%(np.max(np.abs(e_ulp)),np.mean(e_ulp)))
