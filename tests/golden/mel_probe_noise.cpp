// The noise of the reference's mel probe (tests/test_mel_cpu.cpp:55-58 of the
// reference): std::mt19937 seeded 7301, std::uniform_real_distribution<float>
// over [-1, 1), 480,000 draws, written to stdout as raw float32.  Built and run
// by tests/test_audio_oracle.py with the host's g++ and libstdc++.
#include <cstdio>
#include <random>
#include <vector>

int main() {
    const int samples = 480000;
    std::vector<float> noise(samples);
    std::mt19937 rng(7301);
    std::uniform_real_distribution<float> dist(-1, 1);
    for (int n = 0; n < samples; ++n) noise[n] = dist(rng);
    return std::fwrite(noise.data(), sizeof(float), samples, stdout) == (size_t)samples ? 0 : 1;
}
