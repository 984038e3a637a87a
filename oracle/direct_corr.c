/* Test infrastructure: brute-force circular 2D correlation / convolution in
 * double precision -- the definition the FFT path must reproduce
 * (torch.fft.irfftn(rfftn(I) * conj(rfftn(T, s=(H, W)))) of
 * zipFFT tests/test_real_conv_2d.py:110-123 equals this sum).  O(h w oy ox);
 * small sizes only.  Used by tests/ and tests/golden/make_golden.py to pin
 * the FFT oracle; never by the library. */
void direct_corr2d(const double* t, int h, int w, const double* img, int H, int W, int corr,
                   double* out, int oy, int ox) {
    for (int u = 0; u < oy; ++u) {
        for (int v = 0; v < ox; ++v) {
            double acc = 0.0;
            for (int y = 0; y < h; ++y) {
                int iy = corr ? (y + u) % H : ((u - y) % H + H) % H;
                const double* irow = img + (long)iy * W;
                const double* trow = t + (long)y * w;
                for (int x = 0; x < w; ++x) {
                    int ix = corr ? (x + v) % W : ((v - x) % W + W) % W;
                    acc += trow[x] * irow[ix];
                }
            }
            out[(long)u * ox + v] = acc;
        }
    }
}
